/* TEST INFRASTRUCTURE -- the CPU checker, never the product.
 *
 * Plain-C restatement of the reference's packed-wave EmbeddingGemma 2 text
 * graph (vendor/embeddinggemma.c/src/gemma2_fast.c:919-1017) along its scalar
 * code paths, i.e. what the reference computes with EI_GEMMA2_CPU_X86=scalar.
 * Every function cites the reference lines it follows.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU baseline may load this.
 *
 * Parity pin: tests/test_cpu_oracle.py checks that eg2o_embed_batch() is
 * bit-identical to the compiled reference (oracle/_ref/libeg2ref.so, scalar
 * tier) and that the x86 quantizer / GELU variants below are bit-identical to
 * the reference's g2x_* functions on random inputs.
 */
#ifndef EG2_ORACLE_H
#define EG2_ORACLE_H
#include <stddef.h>
#include <stdint.h>

/* Tensor pointer table, in the order of synthetic.tensor_table():
 * 0 token_embd (Q8_0 [262144][512]), 1 per_layer_model_proj (BF16 [12288][512]),
 * 2 per_layer_proj_norm (F32 [512]), then per layer l at 3 + 17*l:
 * attn_norm, attn_q, attn_k, attn_v, attn_output, attn_q_norm, attn_k_norm,
 * post_attention_norm, ffn_norm, ffn_up, ffn_gate, ffn_down, post_ffw_norm,
 * inp_gate, proj, post_norm, layer_output_scale; then output_norm (F32) and
 * output (Q8_0 [768][512]) at 3 + 17*24 and 4 + 17*24. */
#define EG2O_N_TENSORS (3 + 17 * 24 + 2)
enum { EG2O_ROUND_SCALAR = 0, EG2O_ROUND_X86 = 1 };

/* fp32 <-> fp16 (quants.c:13-37, common.h:17-40). */
uint16_t eg2o_fp32_to_fp16(float f);
float eg2o_fp16_to_fp32(uint16_t h);
/* Q8_0 quantization of n floats (n % 32 == 0) into int8 codes qs[n] and fp16
 * scales d[n/32].  mode 0: quants.c:97-177 generic (roundf, clamp);
 * mode 1: gemma2_fast_x86.c:211-234 (trunc(v +- 0.5)). */
void eg2o_quantize(const float *x, int8_t *qs, uint16_t *d, int n, int mode);
/* GELU-tanh times u (u may be NULL).  mode 0: kernels.c:367-371 with tanhf;
 * mode 1: gemma2_fast_x86.c:290-325 (exp8 Cody-Waite polynomial). */
void eg2o_gelu_mul(float *g, const float *u, int n, int mode);
/* y[t][r] = sum_p ((float)dot_p * dw) * dx, p ascending (gemma2_fast.c:193-204). */
void eg2o_gemm_q8(const int8_t *wq, const uint16_t *wd, const int8_t *xq, const uint16_t *xd,
                  int n, int k, int m, float *y);
/* int32 per-block dots D[t][r][p] = sum_z wq[r][32p+z] * xq[t][32p+z]. */
void eg2o_gemm_q8_blockdots(const int8_t *wq, const int8_t *xq, int n, int k, int m, int32_t *D);
/* y[t][r] = sum_z w[r][z] * x[t][z], z ascending; w BF16 (gemma2_fast.c:482-559 scalar). */
void eg2o_gemm_bf16(const uint16_t *w, const float *x, int n, int k, int m, float *y);
/* rms_row (gemma2_fast.c:667-671) with the scalar double sum (gemma2_fast.c:587-590). */
void eg2o_rms_row(float *r, int d, const float *w);
/* RoPE tables, 8192 positions, d = 256 (base 1e4) or 512 (base 1e6) (gemma2_fast.c:116-129). */
void eg2o_rope_tables(int d, float *cos_out, float *sin_out);
/* Packed varlen attention (gemma2_fast.c:768-894 scalar).  q [n][4][d],
 * k, v [n][kv][d], lo/hi per-token sequence bounds, window 512 or 0. */
void eg2o_attention(const float *q, const float *k, const float *v, const uint32_t *lo,
                    const uint32_t *hi, int n, int kv, int d, int window, float *a);

/* The whole graph (gemma2_fast.c:919-1017).  quant_mode selects the Q8 rounding
 * of every activation quantization, gelu_mode the GELU form.  If x_layers is
 * non-NULL it receives the residual stream entering each layer and after the
 * last one, [25][n][512].  Returns 0 on success. */
int eg2o_embed_batch(const void *const *tensors, const int32_t *ids, const size_t *offsets,
                     size_t batch, float *out, int quant_mode, int gelu_mode, float *x_layers);
/* eg2o_embed_batch that also returns the per-layer embedding stream ple_out
 * [n][24][512] (gemma2_fast.c:951-956) beside x_layers (either may be NULL). */
int eg2o_embed_trace(const void *const *tensors, const int32_t *ids, const size_t *offsets, size_t batch,
                     float *out, int quant_mode, int gelu_mode, float *x_layers, float *ple_out);
/* One layer l of the graph (gemma2_fast.c:957-992) on the residual stream x
 * [n][512], in place, with the per-layer embeddings ple [n][24][512] of the
 * same wave (offsets as for eg2o_embed_batch).  Returns 0 on success. */
int eg2o_layer(const void *const *tensors, int l, float *x, const float *ple, const size_t *offsets, size_t batch,
               int quant_mode, int gelu_mode);
/* Test perturbations (default 0, 0): gemm_descending sums each GEMM's Q8_0
 * blocks in descending instead of ascending order (another float order, as
 * the reference's x86 tiers have); attention_fp16 rounds q, k and v to fp16
 * before the attention (the fast path's tensor-core operands).  Used only to
 * measure how far such changes move one layer's output. */
void eg2o_set_variant(int gemm_descending, int attention_fp16);
/* Float order of the GEMMs, PLE projection, sums of squares and attention:
 * EG2O_ORDER_SCALAR (default) the scalar loops; EG2O_ORDER_VNNI512 the
 * reference's default tier on an AVX-512 VNNI host (gemma2_fast_x86.c: lane
 * sums of g2x_gemm512_tile for waves of more than 8 tokens, of
 * q8_tile_vnni512 otherwise; g2x_dot4x4, g2x_sum_squares, g2x_pv).  Combine
 * with the x86 quantizer and GELU for that tier's embeddings. */
enum { EG2O_ORDER_SCALAR = 0, EG2O_ORDER_VNNI512 = 1 };
void eg2o_set_order(int order);
/* The same graph from caller-given 512-wide input rows (media soft tokens,
 * gemma2_fast.c:940-941) instead of token ids.  Returns 0 on success. */
int eg2o_embed_batch_inputs(const void *const *tensors, const float *inputs, const size_t *offsets,
                            size_t batch, float *out, int quant_mode, int gelu_mode);
#endif
