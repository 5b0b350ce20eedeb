/* Test infrastructure only: the reference's own engine
 * (vendor/embeddinggemma.c/src/engine.c, compiled unchanged with
 * -DEI_ENABLE_KFD=1 against this repository's include/, where gemma2_kfd.h
 * forwards to eg2_executor.h) linked with libeg2_b200.so -- the way the
 * reference's CMakeLists.txt:29-40 links gemma2_kfd.cpp into eg2-core.  It
 * proves the drop-in link: the engine's --backend kfd path
 * (engine.c:38-45, ei_gemma2_kfd_create) and its packed-wave path
 * (engine.c:1046-1048, ei_gemma2_kfd_batch) reach the B200 executor.
 * Built by the engine_link target of oracle/Makefile into
 * oracle/_ref/libeg2enginelink.so; loaded by tests only.
 *
 * Entry points wrapped (paths inside p3psi-boo/EmbeddingGemma2-AMDKFD):
 *   ei_engine_load_backend           vendor/embeddinggemma.c/src/engine.c:30
 *   ei_tokenize_spm                  vendor/embeddinggemma.c/src/tokenizer.c (engine.c:1143)
 *   ei_engine_embed_tokens_batch     vendor/embeddinggemma.c/src/engine.c:1021
 *   ei_engine_free                   vendor/embeddinggemma.c/src/engine.c:~205
 */
#include "engine.h"

#include <string.h>

void *eg2link_open(const char *model_path) {
    ei_engine *e = ei_xcalloc(1, sizeof *e);
    ei_engine_load_backend(e, model_path, "kfd");  /* exits with the executor's message on failure */
    return e;
}

/* The engine on its CPU backend (no GPU needed), for its tokenizer. */
void *eg2link_open_cpu(const char *model_path) {
    ei_engine *e = ei_xcalloc(1, sizeof *e);
    ei_engine_load_backend(e, model_path, "cpu");
    return e;
}

/* The engine's own tokenization of a text, as its embed path does it
 * (engine.c:1143: ei_tokenize_spm with the special tokens added); returns the
 * token count and copies up to cap ids. */
size_t eg2link_tokenize(void *h, const char *text, size_t len, int32_t *ids, size_t cap) {
    ei_tokens toks = {0};
    ei_tokenize_spm(&((ei_engine *)h)->tokenizer, text, len, true, false, &toks);
    size_t n = toks.n;
    if (ids) memcpy(ids, toks.ids, (n < cap ? n : cap) * sizeof *ids);
    ei_tokens_free(&toks);
    return n;
}

const char *eg2link_backend(void *h) { return ei_engine_backend((ei_engine *)h); }

int eg2link_embed_batch(void *h, const int32_t *ids, const size_t *offsets, size_t batch, float *out, char *err,
                        size_t err_len) {
    return ei_engine_embed_tokens_batch((ei_engine *)h, ids, offsets, batch, out, err, err_len) ? 1 : 0;
}

void eg2link_close(void *h) {
    if (!h) return;
    ei_engine_free((ei_engine *)h);
    free(h);
}
