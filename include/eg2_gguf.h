/* GGUF model handle shared by the executor ABI.
 *
 * `ei_gguf` / `ei_tensor` / `ei_kv` / `ei_str` below are layout-identical to
 * the reference's vendor/embeddinggemma.c/src/gguf.h:9-60, because
 * `ei_gemma2_kfd_create` (src/gemma2_kfd.h:7) receives the caller's `ei_gguf`
 * produced by the reference's own loader (gguf.c:124 `ei_gguf_open`).  When the
 * reference's gguf.h is included first (EI_GGUF_H defined) its definitions are
 * used instead of these.
 *
 * `eg2_gguf_open` / `eg2_gguf_close` are this library's own loader, for callers
 * that do not link the reference's gguf.c (the Python host and the tests).
 */
#ifndef EG2_GGUF_H
#define EG2_GGUF_H
#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifndef EI_GGUF_H
typedef struct {
    const char *str; /* not null-terminated */
    uint64_t len;
} ei_str;

typedef struct {
    ei_str key;
    uint32_t type;
    union {
        uint64_t u64;
        int64_t i64;
        double f64;
        bool b;
        ei_str s;
    } v;
    uint32_t arr_type;
    uint64_t arr_n;
    const void *arr_data;
} ei_kv;

typedef struct {
    ei_str name;
    uint32_t n_dims;
    uint64_t ne[4]; /* ne[0] = row length */
    uint32_t type;  /* 0 F32, 1 F16, 2 Q4_0, 8 Q8_0, 30 BF16 */
    uint64_t offset;
    const void *data;
    uint64_t n_bytes;
} ei_tensor;

typedef struct {
    const uint8_t *map;
    size_t map_len;
    uint32_t version;
    uint64_t n_kv;
    uint64_t n_tensors;
    uint64_t alignment;
    uint64_t data_off;
    ei_kv *kv;
    ei_tensor *tensors;
} ei_gguf;
#endif

#ifdef __cplusplus
extern "C" {
#endif
/* mmap + index a GGUF v3 file into *g.  Returns false with a message in err.
 * No counterpart in the reference's executor ABI (the reference server links
 * its own loader, vendor/embeddinggemma.c/src/gguf.c:124). */
bool eg2_gguf_open(ei_gguf *g, const char *path, char *err, size_t err_len);
void eg2_gguf_close(ei_gguf *g);
/* sizeof(ei_gguf) as compiled into this library (ABI check for FFI callers). */
size_t eg2_gguf_struct_size(void);
#ifdef __cplusplus
}
#endif
#endif
