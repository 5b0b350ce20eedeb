// All device code of the library, its launchers, and the exported operator
// ABI (include/eg2_ops.h).  Built for sm_100a only.
#include <cstdlib>
#include <mutex>

#include "../../include/eg2_ops.h"
#include "attention.cuh"
#include "attention_tc.cuh"
#include "exact.cuh"
#include "launch.h"
#include "opsabi.cuh"
#include "ple.cuh"
#include "q8gemm.cuh"
#include "q8vnni.cuh"
#include "rowops.cuh"

namespace eg2 {

// ---------------------------------------------------------------- tensor maps
using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiled encode_fn() {
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    });
    return fn;
}

bool encode_tmap_2d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, uint64_t inner, uint64_t outer,
                    uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
    EncodeTiled fn = encode_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) || (row_bytes & 15)) return false;
    const cuuint64_t dims[2] = {inner, outer}, strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer}, estr[2] = {1, 1};
    return fn(map, dtype, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
bool q8_tmap(CUtensorMap *map, const int8_t *base, uint64_t k, uint64_t rows, uint32_t box_rows) {
    return encode_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, base, k, rows, k, 128, box_rows, true);
}
bool bf16_tmap(CUtensorMap *map, const void *base, uint64_t k, uint64_t rows, uint32_t box_rows) {
    return encode_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, k, rows, k * 2, 64, box_rows, true);
}
bool f16_head_tmap(CUtensorMap *map, const void *base, uint64_t d, uint64_t heads, uint64_t n, uint32_t box_rows) {
    EncodeTiled fn = encode_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) || !heads || !n || (d != 256 && d != 512)) return false;
    const cuuint64_t dims[3] = {d, heads, n}, strides[2] = {d * 2, heads * d * 2};
    const cuuint32_t box[3] = {64, 1, box_rows}, estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
bool scale_tmap(CUtensorMap *map, const float *base, uint64_t stride, uint64_t kb, uint32_t box_cols) {
    return encode_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, base, stride, kb, stride * 4, box_cols,
                          uint32_t(kb), false);
}

static int sm_count() {
    static int counts[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!counts[dev]) {
        int c = 0;
        cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
        counts[dev] = c > 0 ? c : 148;
    }
    return counts[dev];
}

// ---------------------------------------------------------------- launchers
// Wave kernels are launched with programmatic stream serialization: a kernel
// may be scheduled while its predecessor still runs; it executes its prologue
// and then blocks in pdl_wait() until the predecessor's results are visible
// (every wave kernel calls pdl_wait() before touching global data).
// EG2_B200_PDL=0 launches them in plain stream order instead.
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid, cfg.blockDim = block, cfg.dynamicSmemBytes = smem, cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    static const bool enabled = [] {
        const char *e = std::getenv("EG2_B200_PDL");
        return !(e && e[0] == '0');
    }();
    cfg.attrs = attr, cfg.numAttrs = enabled ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
template <bool EXACT, bool GEGLU, int TIER = TIER_X86>
static cudaError_t q8gemm_go(const CUtensorMap &w, const CUtensorMap &x, const CUtensorMap &sw,
                             const CUtensorMap &sx, const Q8GemmParams &p, cudaStream_t s) {
    const Q8Smem L = q8gemm_smem(p.K, GEGLU);
    if (L.total > 227 * 1024) return cudaErrorInvalidValue;
    const int grid = p.num_tiles < sm_count() ? p.num_tiles : sm_count();
    return launch_pdl(q8gemm_kernel<EXACT, GEGLU, TIER>, dim3(grid), dim3(Q8Cfg::THREADS), L.total, s, w, x, sw, sx,
                      p);
}
cudaError_t launch_q8gemm(const CUtensorMap &w, const CUtensorMap &x, const CUtensorMap &sw, const CUtensorMap &sx,
                          bool exact, float *out, int ldo, int T, int R, int K, cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    if (K <= 0 || K % 128 || K > 2048 || R <= 0 || R % Q8Cfg::BM || ldo < R) return cudaErrorInvalidValue;
    Q8GemmParams p{out, ldo, T, R, K, (T + Q8Cfg::BN - 1) / Q8Cfg::BN, 0, nullptr, nullptr, 0};
    p.num_tiles = (R / Q8Cfg::BM) * p.tiles_t;
    return exact ? q8gemm_go<true, false>(w, x, sw, sx, p, s) : q8gemm_go<false, false>(w, x, sw, sx, p, s);
}
cudaError_t launch_q8gemm_vnni(const int8_t *wq, const float *ws, const int8_t *xq, const float *xs, int xs_stride,
                               float *out, float *out_up, int ldo, int T, int R, int K, const unsigned *offsets,
                               const unsigned *count, cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    if (!wq || !ws || !xq || !xs || !out || K <= 0 || K % Q8VnniCfg::KC || R <= 0 || R % 128 || xs_stride < T)
        return cudaErrorInvalidValue;
    if (out_up ? ldo < R / 2 : ldo < R) return cudaErrorInvalidValue;
    return launch_pdl(q8gemm_vnni_kernel, dim3(R / Q8VnniCfg::BR, (T + Q8VnniCfg::BT - 1) / Q8VnniCfg::BT),
                      dim3(Q8VnniCfg::THREADS), 0, s, out, out_up, ldo, wq, ws, xq, xs, xs_stride, T, R, K, offsets,
                      count);
}
cudaError_t launch_q8gemm_geglu(const CUtensorMap &w, const CUtensorMap &x, const CUtensorMap &sw,
                                const CUtensorMap &sx, bool exact, int8_t *q8, float *q8s, int q8s_stride, int T, int R,
                                int K, cudaStream_t s, int tier) {
    if (T <= 0) return cudaSuccess;
    if (K <= 0 || K % 128 || K > 2048 || R <= 0 || R % Q8Cfg::BM || q8s_stride < T || !q8 || !q8s)
        return cudaErrorInvalidValue;
    Q8GemmParams p{nullptr, 0, T, R, K, (T + Q8Cfg::BN - 1) / Q8Cfg::BN, 0, q8, q8s, q8s_stride};
    p.num_tiles = (R / Q8Cfg::BM) * p.tiles_t;
    if (tier == TIER_SCALAR)
        return exact ? q8gemm_go<true, true, TIER_SCALAR>(w, x, sw, sx, p, s)
                     : q8gemm_go<false, true, TIER_SCALAR>(w, x, sw, sx, p, s);
    return exact ? q8gemm_go<true, true, TIER_X86>(w, x, sw, sx, p, s)
                 : q8gemm_go<false, true, TIER_X86>(w, x, sw, sx, p, s);
}

cudaError_t launch_ple(const CUtensorMap &hi, const CUtensorMap &lo, const CUtensorMap &w, float *ple,
                       const float *norm, int M, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    const PleParams p{ple, norm, M};
    return launch_pdl(ple_kernel, dim3(24, (M + 127) / 128), dim3(PleCfg::THREADS), PleCfg::SMEM, s, hi, lo, w, p);
}

cudaError_t launch_input_rows(float *x, void *x_hi, void *x_lo, const float *rows, int n, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    return launch_pdl(input_rows_kernel, dim3((unsigned(n) * 512 + 255) / 256), dim3(256), 0, s, x,
                      static_cast<__nv_bfloat16 *>(x_hi), static_cast<__nv_bfloat16 *>(x_lo), rows, n);
}
cudaError_t launch_embed(float *x, void *x_hi, void *x_lo, const void *emb, const int *ids, int n, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    if ((x_hi == nullptr) != (x_lo == nullptr)) return cudaErrorInvalidValue;
    return launch_pdl(embed_kernel, dim3((n + 7) / 8), dim3(256), 0, s, x, static_cast<__nv_bfloat16 *>(x_hi),
                      static_cast<__nv_bfloat16 *>(x_lo), static_cast<const uint8_t *>(emb), ids, n);
}

cudaError_t launch_norm_quant(int8_t *q, float *qs, int qs_stride, float *y, const float *x, const float *w, int rows,
                              int width, cudaStream_t s, int tier) {
    if (rows <= 0) return cudaSuccess;
    if (qs_stride < rows) return cudaErrorInvalidValue;
    if (width != 256 && width != 512 && width != 1024 && width != 2048) return cudaErrorInvalidValue;
    if (!w) {  // ROW_QUANT: no row reduction, warp per (row, four blocks)
        const int warps = rows * (width / 128);
        return launch_pdl(quant_rows_kernel, dim3((warps + 7) / 8), dim3(256), 0, s, q, qs, qs_stride, x, rows, width,
                          tier);
    }
    switch (width) {  // ROW_NORM_QUANT: CTA per row, one float4 per thread
        case 256: return launch_pdl(norm_quant_kernel<256>, dim3(rows), dim3(64), 0, s, q, qs, qs_stride, y, x, w, tier);
        case 512: return launch_pdl(norm_quant_kernel<512>, dim3(rows), dim3(128), 0, s, q, qs, qs_stride, y, x, w, tier);
        case 1024:
            return launch_pdl(norm_quant_kernel<1024>, dim3(rows), dim3(256), 0, s, q, qs, qs_stride, y, x, w, tier);
        default:
            return launch_pdl(norm_quant_kernel<2048>, dim3(rows), dim3(512), 0, s, q, qs, qs_stride, y, x, w, tier);
    }
}

cudaError_t launch_qkv_post(void *q, void *k, void *v, const float *qkv, const float *qn, const float *kn,
                            const float *rc, const float *rs, const unsigned *pos, int n, int d, cudaStream_t s,
                            bool f32_out, int tier) {
    if (n <= 0) return cudaSuccess;
    if (d != 256 && d != 512) return cudaErrorInvalidValue;
    const int rows_per_tok = 4 + 2 * (512 / d), warps = n * rows_per_tok;
    const dim3 grid((warps + 7) / 8), block(256);
    if (f32_out) {
        auto *qf = static_cast<float *>(q), *kf = static_cast<float *>(k), *vf = static_cast<float *>(v);
        if (d == 256)
            return launch_pdl(qkv_post_kernel<256, float>, grid, block, 0, s, qf, kf, vf, qkv, qn, kn, rc, rs, pos, n, tier);
        return launch_pdl(qkv_post_kernel<512, float>, grid, block, 0, s, qf, kf, vf, qkv, qn, kn, rc, rs, pos, n, tier);
    }
    auto *qh = static_cast<__half *>(q), *kh = static_cast<__half *>(k), *vh = static_cast<__half *>(v);
    if (d == 256) return launch_pdl(qkv_post_kernel<256, __half>, grid, block, 0, s, qh, kh, vh, qkv, qn, kn, rc, rs, pos, n, tier);
    return launch_pdl(qkv_post_kernel<512, __half>, grid, block, 0, s, qh, kh, vh, qkv, qn, kn, rc, rs, pos, n, tier);
}

cudaError_t launch_attention_exact(float *out, const float *q, const float *k, const float *v, const unsigned *bounds,
                                   int n, int d, int window, cudaStream_t s, int tier) {
    if (n <= 0) return cudaSuccess;
    if (n > 2048) return cudaErrorInvalidValue;  // key scores of one row live in shared memory
    const bool vnni = tier == TIER_VNNI512;
    const dim3 grid(n, 4), block(128);
    if (d == 256)
        return launch_pdl(vnni ? attention_exact_kernel<256, true> : attention_exact_kernel<256, false>, grid, block, 0,
                          s, out, q, k, v, bounds, n, window);
    if (d == 512)
        return launch_pdl(vnni ? attention_exact_kernel<512, true> : attention_exact_kernel<512, false>, grid, block, 0,
                          s, out, q, k, v, bounds, n, window);
    return cudaErrorInvalidValue;
}

cudaError_t launch_ple_exact(float *ple, const float *x, const void *w, const float *norm, int n, cudaStream_t s,
                             int tier) {
    if (n <= 0) return cudaSuccess;
    const uint16_t *wb = static_cast<const uint16_t *>(w);
    cudaError_t e;
    if (tier == TIER_VNNI512)
        e = launch_pdl(ple_vnni_kernel, dim3(24 * 512 / PleVnniCfg::BR, (n + PleVnniCfg::BT - 1) / PleVnniCfg::BT),
                       dim3(PleVnniCfg::THREADS), 0, s, ple, x, wb, n);
    else
        e = launch_pdl(ple_exact_kernel, dim3(24 * 512 / PleExactCfg::BR, (n + PleExactCfg::BT - 1) / PleExactCfg::BT),
                       dim3(PleExactCfg::THREADS), 0, s, ple, x, wb, n);
    if (e) return e;
    return launch_pdl(ple_norm_kernel, dim3(n * 24), dim3(128), 0, s, ple, norm, tier);
}

template <int D>
static cudaError_t attention_go(const AttnParams &p, cudaStream_t s) {
    const dim3 grid((p.n + AttnCfg<D>::BQ - 1) / AttnCfg<D>::BQ, 4, D / AttnCfg<D>::DV);
    return launch_pdl(attention_kernel<D>, grid, dim3(AttnCfg<D>::THREADS), AttnCfg<D>::SMEM, s, p);
}
cudaError_t launch_attention(float *out, const void *q, const void *k, const void *v, const unsigned *bounds, int n,
                             int d, int window, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    const AttnParams p{out, static_cast<const __half *>(q), static_cast<const __half *>(k),
                       static_cast<const __half *>(v), bounds, n, window};
    if (d == 256) return attention_go<256>(p, s);
    if (d == 512) return attention_go<512>(p, s);
    return cudaErrorInvalidValue;
}

bool attention_tc_maps(AttnTcMaps *m, const void *q, const void *k, const void *v, int n, int d) {
    const uint64_t kv = d == 256 ? 2 : 1;
    m->d = d;
    return n > 0 && f16_head_tmap(&m->q, q, uint64_t(d), 4, uint64_t(n), AttnTcCfg::BQ) &&
           f16_head_tmap(&m->k, k, uint64_t(d), kv, uint64_t(n), AttnTcCfg::BKEY) &&
           f16_head_tmap(&m->v, v, uint64_t(d), kv, uint64_t(n), AttnTcCfg::BKEY);
}
cudaError_t launch_attention_tc(const AttnTcMaps &m, float *out, const unsigned *bounds, int n, int window,
                                cudaStream_t s, int8_t *q, float *qs, int q_stride, int tier) {
    if (n <= 0) return cudaSuccess;
    if (n > ATTN_TC_MAX_TOKENS || window < 0 || (q ? (!qs || q_stride < n) : !out) || (m.d != 256 && m.d != 512))
        return cudaErrorInvalidValue;
    const AttnTcParams p{out, bounds, n, window, q, qs, q_stride, tier == TIER_SCALAR ? TIER_SCALAR : TIER_X86};
    const dim3 grid((n + AttnTcCfg::BQ - 1) / AttnTcCfg::BQ, 4, m.d / 256);
    if (m.d == 512)
        return launch_pdl(attention_tc_kernel<512>, grid, dim3(AttnTcCfgD<512>::THREADS), AttnTcCfgD<512>::SMEM, s,
                          m.q, m.k, m.v, p);
    return launch_pdl(attention_tc_kernel<256>, grid, dim3(AttnTcCfg::THREADS), AttnTcCfg::SMEM, s, m.q, m.k, m.v, p);
}

cudaError_t launch_post_add(float *x, const float *h, const float *w, const float *scale, int8_t *q, float *qs,
                            int qs_stride, const float *next_w, int rows, cudaStream_t s, int tier) {
    if (rows <= 0) return cudaSuccess;
    if (qs_stride < rows) return cudaErrorInvalidValue;
    return launch_pdl(post_add_kernel, dim3(rows), dim3(128), 0, s, x, h, w, scale, q, qs, qs_stride, next_w, tier);
}

cudaError_t launch_gelu_mul(float *g, const float *u, size_t n, cudaStream_t s, int tier) {
    if (n == 0) return cudaSuccess;
    if (!g || (tier != TIER_SCALAR && n % 8)) return cudaErrorInvalidValue;
    const size_t blocks = (n + 255) / 256, cap = size_t(sm_count()) * 16;
    return launch_pdl(tier == TIER_SCALAR ? gelu_mul_kernel<TIER_SCALAR> : gelu_mul_kernel<TIER_X86>,
                      dim3(unsigned(blocks < cap ? blocks : cap)), dim3(256), 0, s, g, u, n);
}

cudaError_t launch_gate_quant(int8_t *q, float *qs, int qs_stride, const float *x, const float *other, int rows,
                              int width, int other_stride, int other_offset, cudaStream_t s, int tier) {
    if (rows <= 0) return cudaSuccess;
    if (width <= 0 || width % 128 || qs_stride < rows || other_stride % 4 || other_offset % 4 ||
        other_offset + width > other_stride)
        return cudaErrorInvalidValue;
    const int warps = rows * (width / 128);
    return launch_pdl(tier == TIER_SCALAR ? gate_quant_kernel<TIER_SCALAR> : gate_quant_kernel<TIER_X86>,
                      dim3((warps + 7) / 8), dim3(256), 0, s, q, qs, qs_stride, x, other, rows, width, other_stride,
                      other_offset);
}

cudaError_t launch_pool_l2(float *out, const float *y, const unsigned *offsets, int batch, int width, cudaStream_t s,
                           const unsigned *count) {
    if (batch <= 0) return cudaSuccess;
    if (width <= 0 || width % 8 || width > 8192) return cudaErrorInvalidValue;
    if (cudaError_t e = launch_pdl(pool_mean_kernel, dim3((width + 31) / 32, batch < POOL_SEQ ? batch : POOL_SEQ),
                                   dim3(256), 0, s, out, y, offsets, width, batch, count))
        return e;
    return launch_pdl(pool_l2_kernel, dim3(batch), dim3(32), 0, s, out, width, batch, count);
}

cudaError_t launch_repack_q8(const void *blocks, int rows, int k, int8_t *codes, float *scales, int scale_stride,
                             cudaStream_t s, int chunk, int phase) {
    const long long nblk = (long long)rows * (k / 32);
    if (nblk <= 0) return cudaSuccess;
    if (chunk < 0 || (chunk > 0 && rows % chunk)) return cudaErrorInvalidValue;
    repack_q8_kernel<<<unsigned((nblk + 255) / 256), 256, 0, s>>>(static_cast<const uint8_t *>(blocks), rows, k, codes,
                                                                  scales, scale_stride, chunk, phase);
    return cudaGetLastError();
}

cudaError_t init_kernel_attributes() {
    cudaError_t e;
    for (auto k : {q8gemm_kernel<false, false>, q8gemm_kernel<true, false>, q8gemm_kernel<false, true, TIER_X86>,
                   q8gemm_kernel<true, true, TIER_X86>, q8gemm_kernel<false, true, TIER_SCALAR>,
                   q8gemm_kernel<true, true, TIER_SCALAR>})
        if ((e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024))) return e;
    if ((e = cudaFuncSetAttribute(ple_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(PleCfg::SMEM)))) return e;
    if ((e = cudaFuncSetAttribute(attention_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  int(AttnCfg<256>::SMEM))))
        return e;
    if ((e = cudaFuncSetAttribute(attention_tc_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  int(AttnTcCfg::SMEM))))
        return e;
    if ((e = cudaFuncSetAttribute(attention_tc_kernel<512>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  int(AttnTcCfgD<512>::SMEM))))
        return e;
    return cudaFuncSetAttribute(attention_kernel<512>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(AttnCfg<512>::SMEM));
}

int read_device_error() {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_error, sizeof(int)) != cudaSuccess) return -1;
    return v;
}
// One bounded wait on a barrier that nothing arrives at: it runs out after its
// limit (about 2 s), records ERR_WAIT_TIMEOUT in the error word and returns, as
// any timed-out wait of the wave kernels would.  For tests of the failure path.
__global__ void wait_timeout_selftest_kernel() {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        bar_init(&bar, 1);
        fence_bar_init();
        wait_bar(&bar, 0, nullptr);
    }
}
cudaError_t read_device_error_async(int *host, cudaStream_t s) {
    return cudaMemcpyFromSymbolAsync(host, g_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
}
void clear_device_error() {
    const int z = 0;
    cudaMemcpyToSymbol(g_error, &z, sizeof(int));
}

}  // namespace eg2

// ---------------------------------------------------------------- operator ABI
using namespace eg2;
static inline cudaStream_t S(void *s) { return static_cast<cudaStream_t>(s); }
static inline int rc(cudaError_t e) { return int(e); }
// Operators used outside the executor opt into their shared memory on first use
// on the current device.
static cudaError_t ensure_attributes() {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e) return e;
    static std::mutex mu;
    static bool done[64] = {};
    std::lock_guard<std::mutex> g(mu);
    if (dev < 64 && done[dev]) return cudaSuccess;
    e = init_kernel_attributes();
    if (!e && dev < 64) done[dev] = true;
    return e;
}

extern "C" {
int eg2_launch_gather(const EgGather *p, void *s) {
    if (!p->n) return 0;
    abi_gather_kernel<<<(p->n * 512 + 255) / 256, 256, 0, S(s)>>>(*p);
    return rc(cudaGetLastError());
}
int eg2_launch_mm(const EgMM *p, void *s) {
    if (!(p->type == 0 || p->type == 1 || p->type == 8 || p->type == 30) || (p->type == 8 && p->k % 32))
        return rc(cudaErrorInvalidValue);
    if (!p->n || !p->m) return 0;
    abi_mm_kernel<<<dim3((p->m + 15) / 16, (p->n + 15) / 16), 256, 0, S(s)>>>(*p);
    return rc(cudaGetLastError());
}
int eg2_launch_norm(const EgNorm *p, void *s) {
    if (!p->rows) return 0;
    abi_norm_kernel<<<p->rows, 32, 0, S(s)>>>(*p);
    return rc(cudaGetLastError());
}
int eg2_launch_rope(const EgRope *p, void *s) {
    if (!p->n) return 0;
    abi_rope_kernel<<<(p->n * p->heads * (p->d / 2) + 255) / 256, 256, 0, S(s)>>>(*p);
    return rc(cudaGetLastError());
}
int eg2_launch_attention(const EgAttention *p, unsigned d, void *s) {
    if (!p->n) return 0;
    if (d == 256) abi_attention_kernel<256><<<p->n * 4, 32, 0, S(s)>>>(*p);
    else if (d == 512) abi_attention_kernel<512><<<p->n * 4, 32, 0, S(s)>>>(*p);
    else return rc(cudaErrorInvalidValue);
    return rc(cudaGetLastError());
}
int eg2_launch_element(const EgElement *p, void *s) {
    if (!p->n) return 0;
    abi_element_kernel<<<(p->n + 255) / 256, 256, 0, S(s)>>>(*p);
    return rc(cudaGetLastError());
}
int eg2_launch_pool(const EgPool *p, void *s) {
    if (!p->batch) return 0;
    abi_pool_kernel<<<(p->batch * 768 + 255) / 256, 256, 0, S(s)>>>(*p);
    return rc(cudaGetLastError());
}
int eg2_launch_norm_residual(const EgNormResidual *p, void *s) {
    if (!p->rows) return 0;
    abi_norm_residual_kernel<<<p->rows, 32, 0, S(s)>>>(*p);
    return rc(cudaGetLastError());
}
int eg2_launch_norm_rope(const EgNormRope *p, void *s) {
    if (!p->rows) return 0;
    abi_norm_rope_kernel<<<p->rows, 32, 0, S(s)>>>(*p);
    return rc(cudaGetLastError());
}

int eg2_launch_embed(const EgEmbed *p, void *s) {
    return rc(launch_embed(p->x, p->x_hi, p->x_lo, p->token_embd, p->ids, int(p->n), S(s)));
}
int eg2_launch_ple_proj(const EgPleProj *p, void *s) {
    if (cudaError_t e = ensure_attributes()) return rc(e);
    if (!p->n) return 0;
    CUtensorMap hi, lo, w;
    if (!bf16_tmap(&hi, p->x_hi, 512, p->n, 128) || !bf16_tmap(&lo, p->x_lo, 512, p->n, 128) ||
        !bf16_tmap(&w, p->weight, 512, 24 * 512, 256))
        return rc(cudaErrorInvalidValue);
    return rc(launch_ple(hi, lo, w, p->ple, p->norm, int(p->n), S(s)));
}
int eg2_launch_norm_quant(const EgNormQuant *p, void *s) {
    return rc(launch_norm_quant(p->q, p->scale, int(p->scale_stride), p->y, p->x, p->weight, int(p->rows),
                                int(p->width), S(s), int(p->tier)));
}
int eg2_launch_q8_mm(const EgQ8MM *p, void *s) {
    if (cudaError_t e = ensure_attributes()) return rc(e);
    if (!p->n) return 0;
    if (p->k % 128 || p->k > 2048 || p->m % 128 || !p->m || p->xs_stride < p->n || p->xs_stride % 4)
        return rc(cudaErrorInvalidValue);
    CUtensorMap w, x, sw, sx;  // weights on the MMA's M side (128 rows), tokens on N (64)
    if (!q8_tmap(&w, p->wq, p->k, p->m, uint32_t(Q8Cfg::BM)) || !q8_tmap(&x, p->xq, p->k, p->n, uint32_t(Q8Cfg::BN)) ||
        !scale_tmap(&sw, p->ws, p->m, p->k / 32, uint32_t(Q8Cfg::BM)) ||
        !scale_tmap(&sx, p->xs, p->xs_stride, p->k / 32, uint32_t(Q8Cfg::BN)))
        return rc(cudaErrorInvalidValue);
    return rc(launch_q8gemm(w, x, sw, sx, p->exact != 0, p->out, int(p->m), int(p->n), int(p->m), int(p->k), S(s)));
}
int eg2_launch_q8_geglu(const EgQ8GeGLU *p, void *s) {
    if (cudaError_t e = ensure_attributes()) return rc(e);
    if (!p->n) return 0;
    if (p->k % 128 || p->k > 2048 || p->m % 64 || !p->m || p->xs_stride < p->n || p->xs_stride % 4 ||
        p->scale_stride < p->n)
        return rc(cudaErrorInvalidValue);
    const unsigned rows = 2 * p->m;  // interleaved gate/up weight rows
    CUtensorMap w, x, sw, sx;
    if (!q8_tmap(&w, p->wq, p->k, rows, uint32_t(Q8Cfg::BM)) || !q8_tmap(&x, p->xq, p->k, p->n, uint32_t(Q8Cfg::BN)) ||
        !scale_tmap(&sw, p->ws, rows, p->k / 32, uint32_t(Q8Cfg::BM)) ||
        !scale_tmap(&sx, p->xs, p->xs_stride, p->k / 32, uint32_t(Q8Cfg::BN)))
        return rc(cudaErrorInvalidValue);
    return rc(launch_q8gemm_geglu(w, x, sw, sx, p->exact != 0, p->q, p->scale, int(p->scale_stride), int(p->n),
                                  int(rows), int(p->k), S(s), int(p->tier)));
}
int eg2_launch_qkv_post(const EgQkvPost *p, void *s) {
    return rc(launch_qkv_post(p->q, p->k, p->v, p->qkv, p->q_norm, p->k_norm, p->rope_cos, p->rope_sin, p->pos,
                              int(p->n), int(p->d), S(s), false));
}
int eg2_launch_attention_exact(const EgAttention *p, unsigned d, void *s) {
    return rc(launch_attention_exact(p->out, p->q, p->k, p->v, p->bounds, int(p->n), int(d), int(p->window), S(s)));
}
int eg2_launch_attention_f16(const EgAttentionF16 *p, void *s) {
    if (cudaError_t e = ensure_attributes()) return rc(e);
    return rc(launch_attention(p->out, p->q, p->k, p->v, p->bounds, int(p->n), int(p->d), int(p->window), S(s)));
}
int eg2_launch_attention_tc(const EgAttentionF16 *p, void *s) {
    if (cudaError_t e = ensure_attributes()) return rc(e);
    if (!p->n) return 0;
    if (p->d != 256 && p->d != 512) return rc(cudaErrorInvalidValue);
    AttnTcMaps m;
    if (!attention_tc_maps(&m, p->q, p->k, p->v, int(p->n), int(p->d))) return rc(cudaErrorInvalidValue);
    return rc(launch_attention_tc(m, p->out, p->bounds, int(p->n), int(p->window), S(s)));
}
int eg2_launch_attention_tc_q8(const EgAttentionQ8 *p, void *s) {
    if (cudaError_t e = ensure_attributes()) return rc(e);
    if (!p->n) return 0;
    if (p->d != 256 && p->d != 512) return rc(cudaErrorInvalidValue);
    AttnTcMaps m;
    if (!attention_tc_maps(&m, p->qh, p->k, p->v, int(p->n), int(p->d))) return rc(cudaErrorInvalidValue);
    return rc(launch_attention_tc(m, nullptr, p->bounds, int(p->n), int(p->window), S(s), p->q, p->qscale,
                                  int(p->scale_stride), int(p->tier)));
}
int eg2_launch_post_add(const EgPostAdd *p, void *s) {
    return rc(launch_post_add(p->x, p->h, p->weight, p->scale, p->q, p->qscale, int(p->scale_stride), p->next_weight,
                              int(p->rows), S(s), int(p->tier)));
}
int eg2_launch_gate_quant(const EgGateQuant *p, void *s) {
    return rc(launch_gate_quant(p->q, p->scale, int(p->scale_stride), p->x, p->other, int(p->rows), int(p->width),
                                int(p->other_stride), int(p->other_offset), S(s), int(p->tier)));
}
int eg2_launch_gelu_mul(const EgGeluMul *p, void *s) {
    return rc(launch_gelu_mul(p->g, p->u, size_t(p->n), S(s), int(p->tier)));
}
int eg2_launch_pool_l2(const EgPoolL2 *p, void *s) {
    return rc(launch_pool_l2(p->out, p->y, p->offsets, int(p->batch), int(p->width), S(s)));
}
int eg2_repack_q8(const void *blocks_dev, unsigned rows, unsigned k, int8_t *codes, float *scales, void *s) {
    if (k % 32) return rc(cudaErrorInvalidValue);
    return rc(launch_repack_q8(blocks_dev, int(rows), int(k), codes, scales, int(rows), S(s)));
}
int eg2_selftest_wait_timeout(void *s) {
    wait_timeout_selftest_kernel<<<1, 32, 0, S(s)>>>();
    return rc(cudaGetLastError());
}
int eg2_read_error(void) { return read_device_error(); }
void eg2_clear_error(void) { clear_device_error(); }
}
