/* Test infrastructure only: a thin C driver around the reference's OWN CPU
 * graph, compiled together with the unmodified reference sources into
 * oracle/_ref/libeg2ref.so (see oracle/Makefile).  Nothing in the product
 * links or loads this file; tests, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference arm use it as the checker and as the timed
 * CPU baseline.
 *
 * Entry points wrapped (reference paths inside p3psi-boo/EmbeddingGemma2-AMDKFD):
 *   ei_gguf_open / ei_gemma2_validate     vendor/embeddinggemma.c/src/gguf.c:124, gemma2.c:30
 *   ei_gemma2_embed_batch_fast_ctx        vendor/embeddinggemma.c/src/gemma2_fast.c:919
 *   ei_gemma2_embed (reference graph)     vendor/embeddinggemma.c/src/gemma2.c:221
 *   ei_thread_pool_create_spin            vendor/embeddinggemma.c/src/parallel.c:165
 *   g2x_level (x86 tier actually used)    vendor/embeddinggemma.c/src/gemma2_fast_x86.c:24
 */
#include "gemma2.h"
#include "gemma2_fast_x86.h"
#include "kernels.h"

typedef struct {
    ei_gguf g;
    ei_thread_pool *pool;
    ei_gemma2_fast *fast;
    int threads;
} eg2ref;

void *eg2ref_open(const char *path, int threads) {
    eg2ref *r = ei_xcalloc(1, sizeof *r);
    ei_gguf_open(&r->g, path);
    ei_gemma2_validate(&r->g);
    r->threads = threads > 0 ? threads : ei_cpu_count();
    r->pool = ei_thread_pool_create_spin(r->threads, 50);
    r->fast = ei_gemma2_fast_create();
    return r;
}

void eg2ref_close(void *h) {
    eg2ref *r = h;
    if (!r) return;
    ei_gemma2_fast_free(r->fast);
    ei_thread_pool_destroy(r->pool);
    ei_gguf_close(&r->g);
    free(r);
}

int eg2ref_threads(void *h) { return ((eg2ref *)h)->threads; }

/* The reference's default CPU graph (packed wave).  out: batch x 768, L2-normalised. */
int eg2ref_embed_fast(void *h, const int32_t *ids, const size_t *offsets, size_t batch, float *out,
                      char *err, size_t err_len) {
    eg2ref *r = h;
    return ei_gemma2_embed_batch_fast_ctx(r->fast, &r->g, r->pool, ids, NULL, offsets, batch, out,
                                          err, err_len) ? 1 : 0;
}

/* The same graph from 512-wide input rows (media soft tokens; ids NULL). */
int eg2ref_embed_fast_inputs(void *h, const float *inputs, const size_t *offsets, size_t batch, float *out,
                             char *err, size_t err_len) {
    eg2ref *r = h;
    return ei_gemma2_embed_batch_fast_ctx(r->fast, &r->g, r->pool, NULL, inputs, offsets, batch, out,
                                          err, err_len) ? 1 : 0;
}

/* The reference's straight single-sequence graph (secondary oracle). */
int eg2ref_embed_reference(void *h, const int32_t *ids, size_t n, float *out, char *err,
                           size_t err_len) {
    eg2ref *r = h;
    return ei_gemma2_embed(&r->g, r->pool, ids, NULL, n, out, err, err_len) ? 1 : 0;
}

/* Matryoshka prefix renormalisation exactly as the server applies it. */
int eg2ref_normalize_prefix(float *embedding, int dims) {
    return ei_embedding_normalize_prefix(embedding, dims) ? 1 : 0;
}

/* The reference's x86 Q8_0 activation quantizer and fp32->fp16 converter,
 * exported for bit-exact pins of the restatement in oracle/eg2_oracle.c. */
void eg2ref_quantize_row_q8_0(const float *x, void *out, int n) {
#if defined(__x86_64__)
    if (g2x_level()) { g2x_quantize_row_q8_0(x, (ei_block_q8_0 *)out, n); return; }
#endif
    ei_quantize_row_q8_0(x, (ei_block_q8_0 *)out, n);
}
uint16_t eg2ref_fp32_to_fp16(float f) { return ei_fp32_to_fp16(f); }
void eg2ref_gelu_mul_row(float *g, const float *u, int n) {
#if defined(__x86_64__)
    if (g2x_level()) { g2x_gelu_mul_row(g, u, n); return; }
#endif
    for (int z = 0; z < n; z++) g[z] = ei_gelu_tanh(g[z]) * (u ? u[z] : 1.0f);
}
float eg2ref_sum_squares(const float *x, int d) {
#if defined(__x86_64__)
    if (g2x_level()) return g2x_sum_squares(x, d);
#endif
    double s = 0;
    for (int z = 0; z < d; z++) s += (double)x[z] * x[z];
    return (float)s;
}

/* 0 scalar, 1 AVX2, 2 AVX-VNNI, 3 AVX-512 VNNI; 1 if the 512-bit repacked GEMM is on. */
int eg2ref_x86_tier(void) { return g2x_level(); }
int eg2ref_x86_wide512(void) { return g2x_gemm512_enabled(); }
