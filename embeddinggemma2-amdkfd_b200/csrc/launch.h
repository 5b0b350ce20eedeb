// Host-side launchers of the sm_100a kernels (internal to the library).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace eg2 {

// Which of the reference's CPU tiers the quantizer rounding and the GELU follow:
// TIER_X86 -- the x86 tiers (gemma2_fast_x86.c), the fast path's choice;
// TIER_SCALAR -- the scalar tier (EI_GEMMA2_CPU_X86=scalar: quants.c rounding,
// kernels.c tanhf GELU), selectable in parity mode;
// TIER_VNNI512 -- the x86 tiers' rounding and GELU, and in parity mode also the
// float orders of the default tier on an AVX-512 VNNI host (lane sums of
// gemma2_fast_x86.c instead of the scalar loops).
enum : int { TIER_X86 = 0, TIER_SCALAR = 1, TIER_VNNI512 = 2 };

// cuTensorMapEncodeTiled through the runtime's driver entry point.
bool encode_tmap_2d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, uint64_t inner, uint64_t outer,
                    uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, bool swizzle128);
// Q8 operand over a row-major int8 buffer [rows][k]: box 128 B x box_rows, 128-byte swizzle.
bool q8_tmap(CUtensorMap *map, const int8_t *base, uint64_t k, uint64_t rows, uint32_t box_rows);
// BF16 operand over [rows][k] bf16: box 64 elements x box_rows, 128-byte swizzle.
bool bf16_tmap(CUtensorMap *map, const void *base, uint64_t k, uint64_t rows, uint32_t box_rows);
// Block-major fp32 scale plane [kb][stride]: box box_cols x kb, no swizzle.
bool scale_tmap(CUtensorMap *map, const float *base, uint64_t stride, uint64_t kb, uint32_t box_cols);

// Kernel launches (all asynchronous on `s`).  `tier` (above) selects the
// quantizer rounding and GELU of the reference tier to reproduce, and the sum
// orders of the row kernels.
// out[T][ldo] = tokens x weight rows.  Maps: weight codes [R][K] with box
// 128 rows, token codes [T][K] with box 64 rows, weight scales [K/32][R] box
// 128, token scales [K/32][stride] box 64.  R must be a multiple of 128.
// exact: the reference scalar tile's rounding order (bit-identical outputs).
cudaError_t launch_q8gemm(const CUtensorMap &w, const CUtensorMap &x, const CUtensorMap &sw, const CUtensorMap &sx,
                          bool exact, float *out, int ldo, int T, int R, int K, cudaStream_t s);
// GeGLU epilogue (ROW_GELU_QUANT fused): the weight is gate/up interleaved in
// 64-row chunks (rows 128c..128c+63 = gate rows 64c.., the next 64 = up rows
// 64c..); writes Q8_0 codes [T][R/2] of gelu(gate) * up and block-major scales.
cudaError_t launch_q8gemm_geglu(const CUtensorMap &w, const CUtensorMap &x, const CUtensorMap &sw,
                                const CUtensorMap &sx, bool exact, int8_t *q8, float *q8s, int q8s_stride, int T, int R,
                                int K, cudaStream_t s, int tier = 0);
// Parity mode at TIER_VNNI512: the GEMM in the float order of the reference's
// default tier on an AVX-512 VNNI host (q8vnni.cuh), on CUDA cores.  Weight
// codes [R][K] with scales [K/32][R], token codes [T][K] with scales
// [K/32][xs_stride]; out[T][ldo].  With out_up set, the weight is the GeGLU
// interleave of launch_q8gemm_geglu and the gate and up columns go to out and
// out_up ([T][ldo] each).  offsets/count (device memory, may be NULL) give the
// wave's real token count, which selects the reference's path (<= 8 tokens:
// its 4-row tile).  K a multiple of 256, R of 128.
cudaError_t launch_q8gemm_vnni(const int8_t *wq, const float *ws, const int8_t *xq, const float *xs, int xs_stride,
                               float *out, float *out_up, int ldo, int T, int R, int K, const unsigned *offsets,
                               const unsigned *count, cudaStream_t s);
cudaError_t launch_ple(const CUtensorMap &hi, const CUtensorMap &lo, const CUtensorMap &w, float *ple,
                       const float *norm, int M, cudaStream_t s);
cudaError_t launch_embed(float *x, void *x_hi, void *x_lo, const void *emb, const int *ids, int n, cudaStream_t s);
// Soft-token waves: x = rows[n][512] as given, plus the bf16 hi/lo split of x.
cudaError_t launch_input_rows(float *x, void *x_hi, void *x_lo, const float *rows, int n, cudaStream_t s);
cudaError_t launch_norm_quant(int8_t *q, float *qs, int qs_stride, float *y, const float *x, const float *w, int rows,
                              int width, cudaStream_t s, int tier = 0);
// q/k/v outputs are fp16, or fp32 when f32_out (parity mode).
cudaError_t launch_qkv_post(void *q, void *k, void *v, const float *qkv, const float *qn, const float *kn,
                            const float *rc, const float *rs, const unsigned *pos, int n, int d, cudaStream_t s,
                            bool f32_out, int tier = 0);
// Parity mode: the reference's attention and PLE orders on CUDA cores -- the
// scalar loops, or with tier TIER_VNNI512 the lane sums of its default tier on
// an AVX-512 VNNI host.
cudaError_t launch_attention_exact(float *out, const float *q, const float *k, const float *v, const unsigned *bounds,
                                   int n, int d, int window, cudaStream_t s, int tier = 0);
cudaError_t launch_ple_exact(float *ple, const float *x, const void *w, const float *norm, int n, cudaStream_t s,
                             int tier = 0);
cudaError_t launch_attention(float *out, const void *q, const void *k, const void *v, const unsigned *bounds, int n,
                             int d, int window, cudaStream_t s);
// The tensor-core attention (d = 256: Q [n][4][256], K/V [n][2][256]; d = 512:
// Q [n][4][512], K/V [n][1][512]), fp16 through 3-D maps (element, head,
// token) whose token extent is n, so rows past n read as zeros.  At most
// ATTN_TC_MAX_TOKENS tokens per launch (the per-tile key-block list then always
// fits).
constexpr int ATTN_TC_MAX_TOKENS = 8192;
struct AttnTcMaps {
    CUtensorMap q, k, v;
    int d = 256;
};
bool attention_tc_maps(AttnTcMaps *m, const void *q, const void *k, const void *v, int n, int d = 256);
// With q set, writes Q8_0 codes [n][4d] and block-major scales [4d/32][q_stride]
// (the row quantizer's output for the same rows) instead of fp32 out.
cudaError_t launch_attention_tc(const AttnTcMaps &m, float *out, const unsigned *bounds, int n, int window,
                                cudaStream_t s, int8_t *q = nullptr, float *qs = nullptr, int q_stride = 0,
                                int tier = 0);
cudaError_t launch_post_add(float *x, const float *h, const float *w, const float *scale, int8_t *q, float *qs,
                            int qs_stride, const float *next_w, int rows, cudaStream_t s, int tier = 0);
cudaError_t launch_gelu_mul(float *g, const float *u, size_t n, cudaStream_t s, int tier = 0);
cudaError_t launch_gate_quant(int8_t *q, float *qs, int qs_stride, const float *x, const float *other, int rows,
                              int width, int other_stride, int other_offset, cudaStream_t s, int tier = 0);
// Mean pool then L2 of `batch` sequences; with count set (device memory), only
// the first *count of them (batch is then an upper bound, the launch grid).
cudaError_t launch_pool_l2(float *out, const float *y, const unsigned *offsets, int batch, int width, cudaStream_t s,
                           const unsigned *count = nullptr);
// chunk > 0: rows interleaved with another matrix in chunk-row blocks, this
// one at position `phase` (0 or 1) of each pair.
cudaError_t launch_repack_q8(const void *blocks, int rows, int k, int8_t *codes, float *scales, int scale_stride,
                             cudaStream_t s, int chunk = 0, int phase = 0);
// Opt every kernel into its shared-memory size on the current device, before
// any graph capture.
cudaError_t init_kernel_attributes();
int read_device_error();
// Enqueues a copy of the error word into host (pinned) memory on stream s.
cudaError_t read_device_error_async(int *host, cudaStream_t s);
void clear_device_error();

}  // namespace eg2
