/* Test infrastructure only: link stand-ins for the reference's CUDA engine of
 * its OTHER model family (embeddinggemma-300m, vendor/embeddinggemma.c/src/
 * engine_cuda.h, implemented by engine_cuda.cu).  engine.c references these
 * when built with -DEI_ENABLE_CUDA, but for an EmbeddingGemma 2 model it takes
 * the gemma2 branch (engine.c:56-74) and never calls them: the text tower then
 * runs through the ei_gemma2_cuda_* entry points, which libeg2_b200.so
 * provides (include/gemma2_cuda.h).  Built into oracle/_ref/eg2server_cuda by
 * the server_cuda target of oracle/Makefile. */
#include <stdio.h>

#include "engine_cuda.h"

void *ei_cuda_engine_create(const ei_model *model, char *err, size_t err_len) {
    (void)model;
    snprintf(err, err_len, "the embeddinggemma-300m CUDA engine is not part of this build");
    return NULL;
}
void ei_cuda_engine_free(void *handle) { (void)handle; }
bool ei_cuda_engine_reserve(void *handle, size_t total_tokens, size_t batch_size, char *err, size_t err_len) {
    (void)handle, (void)total_tokens, (void)batch_size;
    snprintf(err, err_len, "the embeddinggemma-300m CUDA engine is not part of this build");
    return false;
}
bool ei_cuda_engine_embed_tokens(void *handle, const int32_t *ids, size_t n_tokens, float out[EI_N_EMBD], char *err,
                                 size_t err_len) {
    (void)handle, (void)ids, (void)n_tokens, (void)out;
    snprintf(err, err_len, "the embeddinggemma-300m CUDA engine is not part of this build");
    return false;
}
bool ei_cuda_engine_embed_tokens_batch(void *handle, const int32_t *ids, const size_t *offsets, size_t batch_size,
                                       float *out, char *err, size_t err_len) {
    (void)handle, (void)ids, (void)offsets, (void)batch_size, (void)out;
    snprintf(err, err_len, "the embeddinggemma-300m CUDA engine is not part of this build");
    return false;
}
