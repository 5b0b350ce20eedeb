/* Operator ABI: the reference's kernels/abi.h surface plus the fused sm_100a
 * operators the B200 executor is built from.
 *
 * Part 1 keeps the nine parameter structs of kernels/abi.h:3-11 byte for byte
 * and with the semantics of the reference kernels in kernels/eg2.c (fp32
 * activations, GGUF weight types 0/1/8/30, out[n][m] = x[n][k] . W[m][k]^T).
 * Each `eg2_launch_<op>` replaces one `eg2_<op>` code object of
 * kernels/eg2.c and enqueues the operation on a CUDA stream (`stream` is a
 * cudaStream_t, NULL for the default stream); all pointers are device memory.
 * They return 0 or a CUDA error code.
 *
 * Part 2 adds the operators of the executor's fast path (no counterpart in
 * kernels/abi.h; they follow the reference's CPU graph,
 * vendor/embeddinggemma.c/src/gemma2_fast.c, which quantizes activations to
 * Q8_0 before every Q8_0 GEMM):
 *   - Q8 activations are structure-of-arrays: int8 codes [rows][width] and fp32
 *     block scales stored block-major, scale[b * scale_stride + row], whose
 *     values are the fp16 scales the reference stores, widened exactly;
 *   - Q8 weights are the same SoA form, codes [m][k] and scales [k/32][m].
 */
#ifndef EG2_OPS_H
#define EG2_OPS_H
#include <stdint.h>

/* ---- Part 1: kernels/abi.h:3-11, unchanged ---------------------------- */
#ifndef EG2_KFD_ABI_H
typedef struct { float *out; const void *weight; const int *ids; unsigned n; } EgGather;
typedef struct { float *out; const float *x; const void *weight; unsigned n, k, m, type; } EgMM;
typedef struct { float *out; const float *x; const float *weight; unsigned rows, d; float scale; } EgNorm;
typedef struct { float *x; const float *table; unsigned n, heads, d; } EgRope;
typedef struct { float *out; const float *q, *k, *v; const unsigned *bounds; unsigned n, window; } EgAttention;
typedef struct { float *out; const float *x, *other; unsigned n, mode, layer; float scale; } EgElement;
typedef struct { float *out; const float *x; const unsigned *offsets; unsigned batch; } EgPool;
typedef struct { float *out; const float *x, *weight; unsigned rows, d; float scale; } EgNormResidual;
typedef struct { float *x; const float *weight, *table; unsigned rows, d, heads; } EgNormRope;
#endif

/* ---- Part 2: fused sm_100a operators of the executor --------------------- */
/* x[t] = dequant(token_embd[ids[t]]) * sqrt(512) (gemma2_fast.c:942-950), plus
 * the bf16 hi/lo split of x consumed by the PLE tensor-core GEMM (either may
 * be NULL). */
typedef struct { float *x; uint16_t *x_hi, *x_lo; const void *token_embd; const int *ids; unsigned n; } EgEmbed;
/* ple[t][l][:] = rms(x[t] . W_ple[l*512:(l+1)*512]^T / sqrt(512)) * w
 * (gemma2_fast.c:951-956): BF16 weights [12288][512], tcgen05 kind::f16. */
typedef struct { float *ple; const uint16_t *x_hi, *x_lo, *weight; const float *norm; unsigned n; } EgPleProj;
/* Row RMS-norm then Q8_0 quantization (ROW_NORM_QUANT, gemma2_fast.c:685-691);
 * weight NULL: quantization only (ROW_QUANT, :728-730).  y (optional) gets the
 * normalised row.  width is 256, 512, 1024 or 2048. */
typedef struct {
    int8_t *q; float *scale; unsigned scale_stride; float *y;
    const float *x, *weight; unsigned rows, width;
    unsigned tier; /* 0: x86 tiers' quantizer rounding, 1: scalar tier's (roundf) */
} EgNormQuant;
/* out[t][r] = sum_b (int32 dot of block b) * xs[b][t] * ws[b][r]
 * (gemma2_fast.c:242-253): tcgen05 kind::i8, int32 block accumulators in TMEM.
 * k % 128 == 0, k <= 2048, m % 128 == 0, xs_stride >= n and a multiple of 4.
 * exact != 0 rounds like the reference's scalar tile (((float)dot * dw) * dx,
 * then +=), giving bit-identical outputs; exact == 0 fuses the last multiply
 * and add (one rounding fewer). */
typedef struct {
    float *out; const int8_t *xq; const float *xs; unsigned xs_stride;
    const int8_t *wq; const float *ws; unsigned n, k, m, exact;
} EgQ8MM;
/* GeGLU projection with its quantization fused (gemma2_fast.c:978-979 and
 * ROW_GELU_QUANT :714-720): g[t][c] = gelu_tanh(gate[t][c]) * up[t][c] with
 * gate = x . Wg^T and up = x . Wu^T computed as in EgQ8MM, then Q8_0 of g:
 * codes q [n][m], scales scale[b * scale_stride + t].  The weight operand is
 * the two matrices interleaved in 64-row chunks: rows 128c .. 128c+63 of
 * wq/ws are gate rows 64c .., rows 128c+64 .. 128c+127 the up rows 64c ..
 * (2m rows, m % 64 == 0; scales [k/32][2m]).  Identical to EgQ8MM on each
 * half followed by EgGateQuant. */
typedef struct {
    int8_t *q; float *scale; unsigned scale_stride;
    const int8_t *xq; const float *xs; unsigned xs_stride;
    const int8_t *wq; const float *ws; unsigned n, k, m, exact;
    unsigned tier; /* as in EgGateQuant */
} EgQ8GeGLU;
/* Per head RMS (q, k weighted; v plain) and NEOX RoPE from host tables at the
 * token's in-sequence position (ROW_QKV_POST, gemma2_fast.c:692-706).  qkv is
 * the fused projection [n][4d | 512 | 512]; outputs are fp16 [n][heads][d]. */
typedef struct {
    uint16_t *q, *k, *v; const float *qkv, *q_norm, *k_norm, *rope_cos, *rope_sin;
    const unsigned *pos; unsigned n, d;
} EgQkvPost;
/* Bidirectional packed-varlen GQA attention, scale 1, keys in [lo, hi) of the
 * token's sequence, intersected with [t-window, t+window] when window != 0
 * (gemma2_fast.c:768-894).  q [n][4][d], k/v [n][512/d][d] fp16; out fp32
 * [n][4][d]. */
typedef struct {
    float *out; const uint16_t *q, *k, *v; const unsigned *bounds; unsigned n, d, window;
} EgAttentionF16;
/* x = (x + rms(h) * w) * scale (ROW_POST_ADD, gemma2_fast.c:707-713), then the
 * next Q8 operand from the new x: RMS-norm with next_weight and quantize, or
 * (next_weight NULL) plain quantization.  scale is a device pointer (NULL: 1). */
typedef struct {
    float *x; const float *h, *weight, *scale;
    int8_t *q; float *qscale; unsigned scale_stride; const float *next_weight; unsigned rows;
    unsigned tier; /* as in EgNormQuant */
} EgPostAdd;
/* g = gelu_tanh(x[t][z]) * other[t * other_stride + other_offset + z], then Q8
 * (ROW_GELU_QUANT / ROW_PLE_GATE_QUANT, gemma2_fast.c:714-727).  width % 128
 * == 0; other_stride and other_offset multiples of 4. */
typedef struct {
    int8_t *q; float *scale; unsigned scale_stride;
    const float *x, *other; unsigned rows, width, other_stride, other_offset;
    unsigned tier; /* 0: x86 tiers' GELU and rounding, 1: scalar tier's (tanhf, roundf) */
} EgGateQuant;
/* g[z] = gelu_tanh(g[z]) * (u ? u[z] : 1) for z < n, in place: the reference's
 * GELU rows, g2x_gelu_mul_row (gemma2_fast_x86.c:308-325) on the x86 tiers
 * (tier 0; n % 8 == 0, the whole-vector part that the graph uses) and
 * ei_gelu_mul_inplace (kernels.h:26, tanhf form) on the scalar tier (tier 1). */
typedef struct { float *g; const float *u; uint64_t n; unsigned tier; } EgGeluMul;
/* out[s] = L2(mean over the sequence's rows of y) (gemma2_fast.c:1000-1008). */
typedef struct { float *out; const float *y; const unsigned *offsets; unsigned batch, width; } EgPoolL2;

#ifdef __cplusplus
extern "C" {
#endif
/* Part 1 -- each replaces the kernel of the same name in kernels/eg2.c. */
int eg2_launch_gather(const EgGather *p, void *stream);              /* eg2.c:36-39 */
int eg2_launch_mm(const EgMM *p, void *stream);                      /* eg2.c:43-118 */
int eg2_launch_norm(const EgNorm *p, void *stream);                  /* eg2.c:122-133 */
int eg2_launch_rope(const EgRope *p, void *stream);                  /* eg2.c:135-143 */
int eg2_launch_attention(const EgAttention *p, unsigned d, void *stream); /* eg2.c:147-170 */
int eg2_launch_element(const EgElement *p, void *stream);            /* eg2.c:173-179 */
int eg2_launch_pool(const EgPool *p, void *stream);                  /* eg2.c:181-188 */
int eg2_launch_norm_residual(const EgNormResidual *p, void *stream); /* eg2.c:192-202 */
int eg2_launch_norm_rope(const EgNormRope *p, void *stream);         /* eg2.c:204-217 */

/* Part 2 -- executor operators (no counterpart in kernels/abi.h). */
int eg2_launch_embed(const EgEmbed *p, void *stream);
int eg2_launch_ple_proj(const EgPleProj *p, void *stream);
int eg2_launch_norm_quant(const EgNormQuant *p, void *stream);
int eg2_launch_q8_mm(const EgQ8MM *p, void *stream);
int eg2_launch_q8_geglu(const EgQ8GeGLU *p, void *stream);
int eg2_launch_qkv_post(const EgQkvPost *p, void *stream);
int eg2_launch_attention_f16(const EgAttentionF16 *p, void *stream);
/* The same attention on the 5th-generation tensor cores, d = 256 (the
 * sliding-window layers) or 512 (the global layers): S = Q.K^T and O += P.V as
 * tcgen05 MMAs with fp32 accumulators in tensor memory, P in fp16.
 * n <= 8192; other d -> error. */
int eg2_launch_attention_tc(const EgAttentionF16 *p, void *stream);
/* eg2_launch_attention_tc with the Q8_0 quantization of its output rows fused
 * (ROW_QUANT, gemma2_fast.c:728-730): codes q [n][4d], block-major scales
 * qscale [4d/32][scale_stride] (scale_stride >= n), bit-identical to
 * eg2_launch_norm_quant (weight NULL) of the fp32 rows; tier as in EgNormQuant;
 * d = 256 or 512. */
typedef struct {
    int8_t *q; float *qscale; unsigned scale_stride;
    const uint16_t *qh, *k, *v; const unsigned *bounds; unsigned n, window, tier, d;
} EgAttentionQ8;
int eg2_launch_attention_tc_q8(const EgAttentionQ8 *p, void *stream);
/* The reference CPU graph's scalar attention order on fp32 q/k/v
 * (gemma2_fast.c:768-894 scalar branch, the executor's parity mode): one
 * sequential dot per key, softmax with the C library's expf rounding, outputs
 * summed in key order.  EgAttention fields as in Part 1; n <= 2048. */
int eg2_launch_attention_exact(const EgAttention *p, unsigned d, void *stream);
int eg2_launch_post_add(const EgPostAdd *p, void *stream);
int eg2_launch_gate_quant(const EgGateQuant *p, void *stream);
int eg2_launch_gelu_mul(const EgGeluMul *p, void *stream);
int eg2_launch_pool_l2(const EgPoolL2 *p, void *stream);
/* Repack GGUF Q8_0 blocks (34 B, device memory) into the SoA weight operand:
 * codes [rows][k] and fp32 scales [k/32][rows]. */
int eg2_repack_q8(const void *blocks_dev, unsigned rows, unsigned k, int8_t *codes, float *scales, void *stream);
/* Device-side error word of the fast-path kernels (current device): a bounded
 * wait that ran out sets it; 0 means no error.  eg2_clear_error resets it. */
int eg2_read_error(void);
void eg2_clear_error(void);
/* Failure-path self test (no counterpart in the reference): enqueues a kernel
 * whose one bounded wait can never complete, so that after its limit (about
 * 2 s) it sets the error word (1, a timed-out wait) and returns; the GPU and the
 * context stay usable.  Queued before a wave on an executor's stream, it makes
 * that wave fail as a real timeout would. */
int eg2_selftest_wait_timeout(void *stream);
#ifdef __cplusplus
}
#endif
#endif
