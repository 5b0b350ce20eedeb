// GGUF v3 loader filling the reference's ei_gguf layout (include/eg2_gguf.h),
// so FFI callers without the reference's gguf.c can build the handle that
// ei_gemma2_kfd_create takes.  Format: magic "GGUF", version 3, tensor and KV
// counts, KVs, tensor infos, data section aligned to general.alignment
// (vendor/embeddinggemma.c/src/gguf.c:124-205 reads the same layout).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>

#include "../../include/eg2_gguf.h"

namespace {
struct Cursor {
    const uint8_t *p, *end;
    const uint8_t *take(uint64_t n) {
        if (uint64_t(end - p) < n) throw std::runtime_error("truncated GGUF file");
        const uint8_t *r = p;
        p += n;
        return r;
    }
    uint32_t u32() {
        uint32_t v;
        std::memcpy(&v, take(4), 4);
        return v;
    }
    uint64_t u64() {
        uint64_t v;
        std::memcpy(&v, take(8), 8);
        return v;
    }
    ei_str str() {
        ei_str s;
        s.len = u64();
        s.str = reinterpret_cast<const char *>(take(s.len));
        return s;
    }
};
uint64_t scalar_size(uint32_t t) {
    switch (t) {
        case 0: case 1: case 7: return 1;     // u8 i8 bool
        case 2: case 3: return 2;             // u16 i16
        case 4: case 5: case 6: return 4;     // u32 i32 f32
        case 10: case 11: case 12: return 8;  // u64 i64 f64
        default: throw std::runtime_error("unsupported GGUF KV type " + std::to_string(t));
    }
}
uint64_t type_bytes(uint32_t t, uint64_t n) {
    switch (t) {
        case 0: return 4 * n;
        case 1: case 30: return 2 * n;
        case 2: return n / 32 * 18;
        case 8: return n / 32 * 34;
        default: throw std::runtime_error("unsupported GGUF tensor type " + std::to_string(t));
    }
}
bool key_is(const ei_str &s, const char *z) { return s.len == std::strlen(z) && !std::memcmp(s.str, z, s.len); }
}  // namespace

extern "C" size_t eg2_gguf_struct_size(void) { return sizeof(ei_gguf); }

extern "C" void eg2_gguf_close(ei_gguf *g) {
    if (!g) return;
    if (g->kv) {
        for (uint64_t i = 0; i < g->n_kv; i++)
            if (g->kv[i].type == 9 && g->kv[i].arr_type == 8) std::free(const_cast<void *>(g->kv[i].arr_data));
    }
    std::free(g->kv);
    std::free(g->tensors);
    if (g->map) munmap(const_cast<uint8_t *>(g->map), g->map_len);
    std::memset(g, 0, sizeof *g);
}

extern "C" bool eg2_gguf_open(ei_gguf *g, const char *path, char *err, size_t err_len) {
    std::memset(g, 0, sizeof *g);
    try {
        if (!path) throw std::runtime_error("null path");
        const int fd = open(path, O_RDONLY);
        if (fd < 0) throw std::runtime_error(std::string("cannot open ") + path);
        struct stat st;
        if (fstat(fd, &st) != 0 || st.st_size <= 0) {
            close(fd);
            throw std::runtime_error("cannot stat GGUF file");
        }
        g->map_len = size_t(st.st_size);
        void *m = mmap(nullptr, g->map_len, PROT_READ, MAP_PRIVATE, fd, 0);
        close(fd);
        if (m == MAP_FAILED) throw std::runtime_error("mmap failed");
        g->map = static_cast<const uint8_t *>(m);
        Cursor c{g->map, g->map + g->map_len};
        if (c.u32() != 0x46554747u) throw std::runtime_error("not a GGUF file");
        g->version = c.u32();
        if (g->version != 3) throw std::runtime_error("only GGUF v3 is supported");
        g->n_tensors = c.u64();
        g->n_kv = c.u64();
        if (g->n_tensors > (1u << 20) || g->n_kv > (1u << 20)) throw std::runtime_error("implausible GGUF counts");
        g->kv = static_cast<ei_kv *>(std::calloc(g->n_kv ? g->n_kv : 1, sizeof(ei_kv)));
        g->tensors = static_cast<ei_tensor *>(std::calloc(g->n_tensors ? g->n_tensors : 1, sizeof(ei_tensor)));
        if (!g->kv || !g->tensors) throw std::runtime_error("out of memory");
        g->alignment = 32;
        for (uint64_t i = 0; i < g->n_kv; i++) {
            ei_kv &kv = g->kv[i];
            kv.key = c.str();
            kv.type = c.u32();
            if (kv.type == 9) {
                kv.arr_type = c.u32();
                kv.arr_n = c.u64();
                if (kv.arr_type == 8) {
                    if (kv.arr_n > g->map_len / 8) throw std::runtime_error("truncated GGUF file");
                    auto *idx = static_cast<ei_str *>(std::malloc(sizeof(ei_str) * (kv.arr_n ? kv.arr_n : 1)));
                    if (!idx) throw std::runtime_error("out of memory");
                    kv.arr_data = idx;
                    for (uint64_t j = 0; j < kv.arr_n; j++) idx[j] = c.str();
                } else if (kv.arr_type == 9) {
                    throw std::runtime_error("nested GGUF arrays are not supported");
                } else {
                    const uint64_t es = scalar_size(kv.arr_type);
                    if (kv.arr_n > g->map_len / es) throw std::runtime_error("truncated GGUF file");
                    kv.arr_data = c.take(es * kv.arr_n);
                }
            } else if (kv.type == 8) {
                kv.v.s = c.str();
            } else {
                const uint64_t sz = scalar_size(kv.type);
                const uint8_t *p = c.take(sz);
                switch (kv.type) {
                    case 1: kv.v.i64 = int8_t(*p); break;
                    case 3: { int16_t v; std::memcpy(&v, p, 2); kv.v.i64 = v; } break;
                    case 5: { int32_t v; std::memcpy(&v, p, 4); kv.v.i64 = v; } break;
                    case 11: std::memcpy(&kv.v.i64, p, 8); break;
                    case 6: { float v; std::memcpy(&v, p, 4); kv.v.f64 = v; } break;
                    case 12: std::memcpy(&kv.v.f64, p, 8); break;
                    case 7: kv.v.b = *p != 0; break;
                    default: { uint64_t v = 0; std::memcpy(&v, p, sz); kv.v.u64 = v; } break;
                }
            }
            if (key_is(kv.key, "general.alignment")) g->alignment = kv.v.u64;
        }
        if (!g->alignment || (g->alignment & (g->alignment - 1))) throw std::runtime_error("bad GGUF alignment");
        for (uint64_t i = 0; i < g->n_tensors; i++) {
            ei_tensor &t = g->tensors[i];
            t.name = c.str();
            t.n_dims = c.u32();
            if (t.n_dims == 0 || t.n_dims > 4) throw std::runtime_error("bad tensor rank");
            for (int d = 0; d < 4; d++) t.ne[d] = 1;
            for (uint32_t d = 0; d < t.n_dims; d++) t.ne[d] = c.u64();
            t.type = c.u32();
            t.offset = c.u64();
        }
        const uint64_t off = uint64_t(c.p - g->map);
        g->data_off = (off + g->alignment - 1) & ~(g->alignment - 1);
        for (uint64_t i = 0; i < g->n_tensors; i++) {
            ei_tensor &t = g->tensors[i];
            for (int d = 0; d < 4; d++)
                if (t.ne[d] == 0 || t.ne[d] > (uint64_t(1) << 40)) throw std::runtime_error("bad tensor shape");
            const uint64_t n = t.ne[0] * t.ne[1] * t.ne[2] * t.ne[3];
            if ((t.type == 2 || t.type == 8) && t.ne[0] % 32) throw std::runtime_error("quantized row not a multiple of 32");
            t.n_bytes = type_bytes(t.type, n);
            if (t.offset % g->alignment) throw std::runtime_error("misaligned tensor offset");
            if (t.offset > g->map_len || g->data_off + t.offset + t.n_bytes > g->map_len)
                throw std::runtime_error("tensor past end of file");
            t.data = g->map + g->data_off + t.offset;
        }
        return true;
    } catch (const std::exception &e) {
        if (err && err_len) std::snprintf(err, err_len, "GGUF: %s", e.what());
        eg2_gguf_close(g);
        return false;
    }
}
