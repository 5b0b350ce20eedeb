/* Test infrastructure only: a thin C driver around the reference's OWN CUDA
 * executor for the same text graph (vendor/embeddinggemma.c/src/gemma2_cuda.cu:
 * fp16 weight copies, cuBLAS GemmEx fp16 x fp16 -> fp32 GEMMs at :593-600,
 * mma.sync flash attention at :327-523, one CUDA graph per wave shape at
 * :749-779), compiled from the reference's sources into
 * oracle/_ref/libeg2cudaref.so (see the cuda_ref target of oracle/Makefile).
 * It is the GPU comparator that bench.py times beside the B200 executor on the
 * same seeded GGUF and token ids; nothing in the product links or loads it.
 *
 * Entry points wrapped (paths inside p3psi-boo/EmbeddingGemma2-AMDKFD):
 *   ei_gguf_open / ei_gguf_close        vendor/embeddinggemma.c/src/gguf.c
 *   ei_gemma2_cuda_create_on            vendor/embeddinggemma.c/src/gemma2_cuda.cu:1330
 *   ei_gemma2_cuda_batch                vendor/embeddinggemma.c/src/gemma2_cuda.cu:1451
 *   ei_gemma2_cuda_free                 vendor/embeddinggemma.c/src/gemma2_cuda.cu:1426
 *   ei_gemma2_cuda_clone                vendor/embeddinggemma.c/src/gemma2_cuda.cu:1490
 */
#include "gemma2_cuda.h"
#include "common.h"

typedef struct {
    ei_gguf g;
    void *ctx;
} eg2cref;

void *eg2cref_open(const char *path, int device, char *err, size_t err_len) {
    eg2cref *r = ei_xcalloc(1, sizeof *r);
    ei_gguf_open(&r->g, path);
    r->ctx = ei_gemma2_cuda_create_on(&r->g, device, err, err_len);
    if (!r->ctx) {
        ei_gguf_close(&r->g);
        free(r);
        return NULL;
    }
    return r;
}

void eg2cref_close(void *h) {
    eg2cref *r = h;
    if (!r) return;
    ei_gemma2_cuda_free(r->ctx);
    ei_gguf_close(&r->g);
    free(r);
}

/* The reference executor's packed-wave call: host ids/offsets in, batch x 768
 * L2-normalised embeddings out, synchronous (uploads, graph, download). */
int eg2cref_batch(void *h, const int32_t *ids, const size_t *offsets, size_t batch, float *out, char *err,
                  size_t err_len) {
    eg2cref *r = h;
    return ei_gemma2_cuda_batch(r->ctx, ids, offsets, batch, out, err, err_len) ? 1 : 0;
}

/* A pipeline slot of the reference executor (its own stream, cuBLAS handle and
 * workspace over the parent's weights), as the reference's engine makes one
 * per extra slot (engine.c:1213-1216); batch and free take the slot itself. */
void *eg2cref_slot(void *h, char *err, size_t err_len) {
    return ei_gemma2_cuda_clone(((eg2cref *)h)->ctx, true, err, err_len);
}
int eg2cref_slot_batch(void *slot, const int32_t *ids, const size_t *offsets, size_t batch, float *out, char *err,
                       size_t err_len) {
    return ei_gemma2_cuda_batch(slot, ids, offsets, batch, out, err, err_len) ? 1 : 0;
}
void eg2cref_slot_free(void *slot) { ei_gemma2_cuda_free(slot); }
