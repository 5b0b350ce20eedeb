/* Drop-in for the reference's CUDA executor ABI, vendor/embeddinggemma.c/src/
 * gemma2_cuda.h:13-33 (implemented by gemma2_cuda.cu:1316-1510 with cuBLAS):
 * the same ten entry points, served by this library's B200 executor, so the
 * reference's engine and server built with -DEI_ENABLE_CUDA (this directory
 * first on the include path) run their CUDA backend -- several devices
 * (--cuda-devices) and pipeline slots (--pipeline-slots) included -- on it.
 *
 *   - create / create_on: a context on EI_CUDA_DEVICE (default 0) or on the
 *     given device, taking waves of up to 8192 packed tokens like the
 *     reference's (gemma2_cuda.cu:717); `g` is borrowed;
 *   - clone: a pipeline slot sharing the parent's weights; the parent must
 *     outlive it.  A context already runs two calls' waves at once on its two
 *     lanes, so a clone is a second handle onto the same context (the
 *     high_priority hint is accepted and not used);
 *   - batch: as ei_gemma2_kfd_batch, waves above 8192 tokens split at
 *     sequence boundaries as gemma2_cuda.cu:1451-1468 does; errors without the
 *     "KFD: " prefix, as the reference's CUDA executor reports them;
 *   - embed_inputs: one sequence of 512-wide input rows (media soft tokens);
 *   - vision / audio: the image and audio towers are not part of this
 *     executor; they fail with a message (their 512-wide outputs are accepted
 *     by embed_inputs and eg2_b200_batch_rows).
 * The embeddings are this executor's (int8 Q8_0 GEMMs with exact block sums),
 * not the reference CUDA executor's fp16 cuBLAS ones. */
#ifndef EG2_GEMMA2_CUDA_H
#define EG2_GEMMA2_CUDA_H
#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>
#include "eg2_gguf.h"
#ifdef __cplusplus
extern "C" {
#endif
void *ei_gemma2_cuda_create(const ei_gguf *g, char *err, size_t len);
void *ei_gemma2_cuda_create_on(const ei_gguf *g, int device, char *err, size_t len);
int ei_gemma2_cuda_device_count(void);
int ei_gemma2_cuda_device(void *ctx);
void ei_gemma2_cuda_free(void *ctx);
void *ei_gemma2_cuda_clone(void *ctx, bool high_priority, char *err, size_t len);
bool ei_gemma2_cuda_batch(void *ctx, const int32_t *ids, const size_t *offsets, size_t batch, float *out,
                          char *err, size_t len);
bool ei_gemma2_cuda_embed_inputs(void *ctx, const float *inputs, size_t n, float out[768], char *err,
                                 size_t len);
bool ei_gemma2_cuda_vision(void *ctx, const ei_gguf *projector, const uint8_t *rgb, int width, int height,
                           float **out, size_t *tokens, char *err, size_t len);
bool ei_gemma2_cuda_audio(void *ctx, const ei_gguf *projector, const float *mel, int frames, float **out,
                          size_t *tokens, char *err, size_t len);
#ifdef __cplusplus
}
#endif
#endif
