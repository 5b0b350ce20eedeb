/* EmbeddingGemma 2 packed-wave executor on NVIDIA B200 (sm_100a).
 *
 * Drop-in for the reference's executor C ABI, src/gemma2_kfd.h:7-10
 * (implemented at src/gemma2_kfd.cpp:358-366), with the same argument meaning,
 * ownership and error behaviour:
 *   - `g` is borrowed and must outlive the context;
 *   - ids / offsets / out are caller-owned HOST memory; `out` receives
 *     batch x 768 floats, already L2-normalised;
 *   - offsets[0] == 0, strictly increasing, 1..2048 packed tokens, token ids in
 *     [0, 262144); violations fail with the reference's messages;
 *   - synchronous: returns after the embeddings are on the host;
 *   - errors return NULL / false with "KFD: <reason>" written into err, as the
 *     reference does (the engine turns that into HTTP 400);
 *   - after a device failure or timeout the context is poisoned and every later
 *     call fails with "... restart process before reuse";
 *   - a kernel's bounded wait that runs out (about 2 s) sets an error word
 *     that is per DEVICE, shared by every context on it: it fails the next
 *     wave of each of them, and creating a context does not clear it;
 *   - calls from several threads are safe: the context's mutex is held only
 *     to enqueue a wave and to deliver it, so two calls' waves run at once on
 *     the context's two lanes (a third waits for a lane).
 */
#ifndef EG2_EXECUTOR_H
#define EG2_EXECUTOR_H
#include "eg2_gguf.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Replaces src/gemma2_kfd.h:7.  Uses CUDA device 0, or EG2_B200_DEVICE. */
void *ei_gemma2_kfd_create(const ei_gguf *g, char *err, size_t len);
/* Replaces src/gemma2_kfd.h:8. */
void ei_gemma2_kfd_free(void *ctx);
/* Replaces src/gemma2_kfd.h:9-10. */
bool ei_gemma2_kfd_batch(void *ctx, const int32_t *ids, const size_t *offsets, size_t batch,
                         float *out, char *err, size_t len);

/* One executor per GPU: the counterpart of the CUDA backend's per-device
 * create (vendor/embeddinggemma.c/src/gemma2_cuda.h:14), which the engine's
 * one-executor-per-device routing (engine.c:1199-1220) needs. */
void *ei_gemma2_kfd_create_on(const ei_gguf *g, int device, char *err, size_t len);

/* ei_gemma2_kfd_create_on with options.  EG2_B200_EXACT selects parity mode:
 * every operation in the reference CPU graph's own float order (GEMMs in the
 * scalar tile's rounding, attention and the PLE projection on exact-order
 * CUDA-core kernels instead of the fp16/bf16 tensor-core ones), for checking
 * results against the reference; about 12x slower.  No counterpart in the
 * reference's executor ABI. */
#define EG2_B200_EXACT 1u
/* With EG2_B200_EXACT: the quantizer rounding (roundf) and GELU (tanhf) of the
 * reference's scalar CPU tier (EI_GEMMA2_CPU_X86=scalar) instead of the x86
 * tiers' (trunc(x +- 0.5), exp polynomial), which the fast path uses. */
#define EG2_B200_SCALAR_TIER 2u
/* With EG2_B200_EXACT: the float orders of the reference CPU graph's default
 * tier on an AVX-512 VNNI host (vnni512 with the repacked 512-bit GEMM,
 * gemma2_fast_x86.c:24-48: its GEMM lane sums, g2x_dot4x4 for the PLE
 * projection and attention scores, g2x_sum_squares, g2x_pv), with its x86
 * quantizer and GELU, so that a wave equals ei_gemma2_embed_batch_fast_ctx on
 * such a host bit for bit.  Excludes EG2_B200_SCALAR_TIER. */
#define EG2_B200_VNNI512_TIER 8u
/* Waves of up to 8192 packed tokens, the reference CPU graph's limit
 * (gemma2_fast.c:924-925, "EmbeddingGemma 2 accepts 1..8192 input tokens")
 * instead of the KFD executor's 2048; the context allocates for 8192 tokens.
 * Fast path only: with EG2_B200_EXACT creation fails. */
#define EG2_B200_WAVE_8192 4u
void *eg2_b200_create(const ei_gguf *g, int device, unsigned flags, char *err, size_t len);

/* The host-side checks of src/gemma2_kfd.cpp:270-278 alone (offsets, token
 * count, id range), with the same messages; no device work.  true = valid. */
bool eg2_b200_validate(const int32_t *ids, const size_t *offsets, size_t batch, char *err, size_t len);

/* ---- split form of ei_gemma2_kfd_batch (same validation and kernels) ------
 * stage: validate, build per-token bounds/positions, copy ids and tables to
 *        the device and select (capturing on first use) the CUDA graph for
 *        this wave shape;
 * launch: replay that graph `repeats` times on the context stream (no sync);
 * finish: wait (with the reference's 30 s deadline), copy the embeddings to
 *        `out` and check them (finite, non-zero).
 * Used by benchmarks to time the device work with inputs already resident.
 * No counterpart in the reference (its batch call is monolithic). */
bool eg2_b200_stage(void *ctx, const int32_t *ids, const size_t *offsets, size_t batch, char *err,
                    size_t len);
bool eg2_b200_launch(void *ctx, int repeats, char *err, size_t len);
bool eg2_b200_finish(void *ctx, float *out, char *err, size_t len);
/* Pipelined form of ei_gemma2_kfd_batch with two slots (the role of the
 * reference server's per-GPU pipeline slots, inference_service.c): submit
 * validates and stages the wave, enqueues its upload, graph and readback, and
 * returns the slot index (or -1 with err set); collect waits for that slot with
 * the batch call's deadline and checks and copies its batch x 768 embeddings.
 * Submits alternate between the two slots; a slot must be collected before it
 * is submitted to again, so the host can prepare or post-process one wave while
 * the GPU runs the other.  Same validation and errors as ei_gemma2_kfd_batch. */
int eg2_b200_submit(void *ctx, const int32_t *ids, const size_t *offsets, size_t batch, char *err, size_t len);
bool eg2_b200_collect(void *ctx, int slot, float *out, char *err, size_t len);
/* ---- media soft-token waves ----------------------------------------------
 * The same wave from caller-given 512-wide input rows instead of token ids:
 * rows [offsets[batch]][512] fp32 become the residual stream x as given, the
 * role of ids == NULL in the reference's CPU graph
 * (ei_gemma2_embed_batch_fast_ctx, gemma2_fast.c:940-941; gemma2.h:10-16).
 * Offsets are checked as for ids (same messages); the rows are not inspected.
 * batch_rows is the monolithic call, stage_rows the split form's first step
 * (then eg2_b200_launch / eg2_b200_finish), submit_rows the pipelined form's
 * (then eg2_b200_collect).  The KFD executor has no counterpart. */
bool eg2_b200_validate_rows(const float *rows, const size_t *offsets, size_t batch, char *err, size_t len);
bool eg2_b200_batch_rows(void *ctx, const float *rows, const size_t *offsets, size_t batch, float *out,
                         char *err, size_t len);
bool eg2_b200_stage_rows(void *ctx, const float *rows, const size_t *offsets, size_t batch, char *err,
                         size_t len);
int eg2_b200_submit_rows(void *ctx, const float *rows, const size_t *offsets, size_t batch, char *err,
                         size_t len);
/* Teacher-forced layer range: layers [first_layer, last_layer) of the
 * context's graph (0 <= first <= last <= 24) run on a caller-given residual
 * stream x_in [offsets[batch]][512] fp32 and per-layer embeddings ple_in
 * [offsets[batch]][24][512] fp32 (NULL: projected on the device from x_in,
 * which must then be the wave's embedding rows), with the wave's sequence
 * bounds and positions from offsets (checked as for ids).  x_out receives the
 * residual stream after layer last_layer - 1.  The reference CPU graph's
 * layer loop (gemma2_fast.c:957-992) has no entry point of its own; this one
 * lets each layer be checked against it from identical inputs.  Synchronous;
 * host memory; replaces the staged wave, if any. */
bool eg2_b200_forward_layers(void *ctx, const float *x_in, const float *ple_in, const size_t *offsets, size_t batch,
                             int first_layer, int last_layer, float *x_out, char *err, size_t len);
/* Matryoshka truncation of one embedding as the reference server applies it
 * (kernels.c:398-407 ei_embedding_normalize_prefix, server.c:1133): keeps the
 * first dims in {128, 256, 512, 768} of the 768 floats and, when shorter,
 * L2-renormalises them in place in the server's summation order.  Host only,
 * thread-safe; false for other dims. */
bool eg2_b200_normalize_prefix(float *embedding, int dims);
/* The cudaStream_t the context launches on (for CUDA-event timing). */
void *eg2_b200_stream(void *ctx);
/* Kernels launched per wave by the staged graph. */
/* Capture the CUDA graphs of every wave shape (64-token buckets of token-id
 * waves) up to max_tokens on both lanes now, instead of on the first wave of
 * each shape (a capture costs milliseconds).  Returns the number of graphs
 * the context holds, or -1 with "KFD: ..." in err.  Setting
 * EG2_B200_PREPARE_TOKENS=n in the environment does the same at context
 * creation, for callers that cannot make this call.  No counterpart in the
 * reference's executor ABI. */
int eg2_b200_prepare(void *ctx, unsigned max_tokens, char *err, size_t len);
int eg2_b200_kernels_per_wave(void *ctx);
/* Time one eager replay of the staged wave per kernel group with CUDA events
 * (the counterpart of EG2_KFD_PROFILE, gemma2_kfd.cpp:173-186,346-352).
 * names/ms receive up to `max` entries; returns the number written, -1 on error. */
int eg2_b200_profile(void *ctx, char names[][32], double *ms, int max);
/* Device the context runs on. */
int eg2_b200_device(void *ctx);

#ifdef __cplusplus
}
#endif
#endif
