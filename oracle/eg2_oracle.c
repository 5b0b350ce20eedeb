/* TEST INFRASTRUCTURE -- the CPU checker, never the product.
 *
 * Restatement of the reference's packed-wave EmbeddingGemma 2 graph along its
 * scalar paths (EI_GEMMA2_CPU_X86=scalar).  Reference files are cited by their
 * path inside p3psi-boo/EmbeddingGemma2-AMDKFD under
 * vendor/embeddinggemma.c/src/.  Built with -std=c11 -O2 (no FMA contraction),
 * like the reference, so that every float operation happens in the same order
 * and rounds the same way.
 */
#include "eg2_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* Runs fn(ctx, lo, hi) over [0, n) split into contiguous ranges, one per host
 * thread (at most 64).  Only independent iterations (tokens, weight rows) are
 * split, so every result is computed in the same order as a serial loop and
 * does not depend on the thread count. */
typedef void (*range_fn)(void *ctx, int lo, int hi);
typedef struct {
    range_fn fn;
    void *ctx;
    int lo, hi;
} range_job;
static void *range_main(void *p) {
    range_job *j = p;
    j->fn(j->ctx, j->lo, j->hi);
    return NULL;
}
static void par_for(int n, range_fn fn, void *ctx) {
    long cpus = sysconf(_SC_NPROCESSORS_ONLN);
    int T = cpus < 1 ? 1 : cpus > 64 ? 64 : (int)cpus;
    if (T > n) T = n;
    if (T <= 1) {
        if (n > 0) fn(ctx, 0, n);
        return;
    }
    pthread_t th[64];
    range_job jobs[64];
    for (int i = 0; i < T; i++) {
        jobs[i] = (range_job){fn, ctx, (int)((long)n * i / T), (int)((long)n * (i + 1) / T)};
        if (i && pthread_create(&th[i], NULL, range_main, &jobs[i])) jobs[i].fn = NULL;
    }
    fn(ctx, jobs[0].lo, jobs[0].hi);
    for (int i = 1; i < T; i++) {
        if (jobs[i].fn) pthread_join(th[i], NULL);
        else fn(ctx, jobs[i].lo, jobs[i].hi);  /* thread creation failed: run it here */
    }
}

/* quants.c:13-37 -- fp32 -> fp16, ties resolved upward on bit 12 (not RNE). */
uint16_t eg2o_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u, mant = x & 0x7FFFFFu;
    int32_t exp = (int32_t)((x >> 23) & 0xFFu) - 112;
    if (exp <= 0) {
        if (exp < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        uint32_t shift = (uint32_t)(14 - exp), half = sign | (mant >> shift);
        if ((mant >> (shift - 1u)) & 1u) half++;
        return (uint16_t)half;
    }
    if (exp >= 31) return (uint16_t)(sign | 0x7C00u | (mant ? ((mant >> 13) | 1u) : 0u));
    uint32_t half = sign | ((uint32_t)exp << 10) | (mant >> 13);
    if (mant & 0x1000u) half++;
    return (uint16_t)half;
}

/* common.h:17-40 -- exact fp16 -> fp32 including subnormals. */
float eg2o_fp16_to_fp32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu, bits;
    if (exp == 0) {
        if (!man) bits = sign;
        else {
            int e = -1;
            uint32_t m = man;
            do { m <<= 1; e++; } while (!(m & 0x400u));
            bits = sign | ((uint32_t)(112 - e) << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (exp == 0x1F) bits = sign | 0x7F800000u | (man << 13);
    else bits = sign | ((exp + 112) << 23) | (man << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static float bf16_to_fp32(uint16_t b) {
    uint32_t bits = (uint32_t)b << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* quants.c:97-177 (generic branch) and gemma2_fast_x86.c:211-234. */
void eg2o_quantize(const float *x, int8_t *qs, uint16_t *dout, int n, int mode) {
    for (int b = 0; b < n / 32; b++) {
        const float *xb = x + b * 32;
        float amax = 0.0f;
        for (int j = 0; j < 32; j++) {
            float a = fabsf(xb[j]);
            if (a > amax) amax = a;
        }
        float d = amax / 127.0f;
        dout[b] = eg2o_fp32_to_fp16(d);
        if (mode == EG2O_ROUND_SCALAR) {
            if (amax == 0.0f) {
                memset(qs + b * 32, 0, 32);
                continue;
            }
            float id = 1.0f / d;
            for (int j = 0; j < 32; j++) {
                int q = (int)roundf(xb[j] * id);
                qs[b * 32 + j] = (int8_t)(q < -128 ? -128 : q > 127 ? 127 : q);
            }
        } else {
            float id = d != 0.0f ? 1.0f / d : 0.0f;
            for (int j = 0; j < 32; j++) {
                float v = xb[j] * id;
                float t = v + copysignf(0.5f, v);
                int q = (int)t; /* cvttps: truncation toward zero */
                qs[b * 32 + j] = (int8_t)(q < -128 ? -128 : q > 127 ? 127 : q);
            }
        }
    }
}

/* gemma2_fast_x86.c:291-306 -- exp via Cody-Waite reduction + degree-6 polynomial. */
static float exp8_lane(float x) {
    x = fminf(fmaxf(x, -87.0f), 88.0f);
    float n = rintf(x * 1.44269504088896341f);
    float r = fmaf(-n, 0.693359375f, x);
    r = fmaf(-n, -2.12194440e-4f, r);
    float p = 1.0f / 720;
    p = fmaf(p, r, 1.0f / 120);
    p = fmaf(p, r, 1.0f / 24);
    p = fmaf(p, r, 1.0f / 6);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    uint32_t e = (uint32_t)((int32_t)n + 127) << 23;
    float s;
    memcpy(&s, &e, 4);
    return p * s;
}

/* kernels.c:367-371 (mode 0) and gemma2_fast_x86.c:308-325 (mode 1). */
void eg2o_gelu_mul(float *g, const float *u, int n, int mode) {
    for (int z = 0; z < n; z++) {
        float x = g[z], gl;
        if (mode == 0 || (n % 8 && z >= n / 8 * 8)) {
            gl = 0.5f * x * (1.0f + tanhf(0.79788456080286535587989211986876f * x * (1.0f + 0.044715f * x * x)));
        } else {
            float inner = (0.79788456080286535588f * x) * fmaf(0.044715f * x, x, 1.0f);
            inner = fminf(fmaxf(inner, -9.0f), 9.0f);
            float t = 1.0f - 2.0f / (exp8_lane(2.0f * inner) + 1.0f);
            gl = (0.5f * x) * (1.0f + t);
        }
        g[z] = gl * (u ? u[z] : 1.0f);
    }
}

/* Perturbations for the tests that measure how far an implementation in
 * another float order can land from this one (never set otherwise): the GEMM
 * sums its blocks in descending order, and/or q, k, v are rounded to fp16
 * before the attention. */
static int variant_gemm_descending, variant_attention_fp16;
void eg2o_set_variant(int gemm_descending, int attention_fp16) {
    variant_gemm_descending = gemm_descending;
    variant_attention_fp16 = attention_fp16;
}

/* Float orders: EG2O_ORDER_SCALAR follows the scalar loops, EG2O_ORDER_VNNI512
 * the reference's default tier on an AVX-512 VNNI host (g2x_level() ==
 * G2X_VNNI512 with the repacked 512-bit GEMM, gemma2_fast_x86.c:24-48). */
static int order_vnni;
void eg2o_set_order(int order) { order_vnni = order == EG2O_ORDER_VNNI512; }

/* Horizontal sum of 8 lanes as hsum / G2X_Q8_TILE end it
 * (gemma2_fast_x86.c:239-244, :95-101): (a_j + a_{j+4}) for j < 4, then
 * (s0 + s2) + (s1 + s3). */
static float hsum8(const float *a) {
    float s0 = a[0] + a[4], s1 = a[1] + a[5], s2 = a[2] + a[6], s3 = a[3] + a[7];
    return (s0 + s2) + (s1 + s3);
}
/* _mm512_reduce_add_ps as the C compiler expands it (gemma2_fast_x86.c:203):
 * the upper and lower 256-bit halves added lane by lane, then the same for
 * 128-bit halves, then lanes 0+2 and 1+3, then those two. */
static float reduce16(const float *a) {
    float t[8], u[4];
    for (int i = 0; i < 8; i++) t[i] = a[i] + a[i + 8];
    for (int i = 0; i < 4; i++) u[i] = t[i] + t[i + 4];
    return (u[0] + u[2]) + (u[1] + u[3]);
}

/* gemma2_fast.c:193-204 -- scalar Q8_0 x Q8_0 tile, blocks in ascending order. */
typedef struct {
    const int8_t *wq, *xq;
    const float *wd, *xd;  /* the fp16 scales, widened exactly */
    int k, m;
    float *y;
    int32_t *D;
    int n;
} gemm_q8_job;
/* gemma2_fast_x86.c:168-204 (g2x_gemm512_tile, waves of more than 8 tokens):
 * 16 fp32 lanes per output, lanes 0-7 taking the int32 sums of bytes 4g..4g+3
 * of block p and lanes 8-15 those of block p + 1, with u8 activations q + 128
 * and lane 0 of each block seeded with -128 * sum(w) (:146-158); each lane
 * adds float(sum) * (sw * sx) with one fused multiply-add per block pair,
 * then _mm512_reduce_add_ps.  gemma2_fast.c:446-465 selects it. */
static float q8_dot_vnni512(const int8_t *w, const int8_t *x, const float *wd, const float *xd, int kb) {
    float acc[16] = {0};
    for (int p = 0; p < kb; p += 2)
        for (int lane = 0; lane < 16; lane++) {
            const int b = p + lane / 8, g = lane % 8;
            const int8_t *wb = w + (size_t)b * 32, *xb = x + (size_t)b * 32;
            int sum = 0;
            for (int i = 4 * g; i < 4 * g + 4; i++) sum += (xb[i] + 128) * wb[i];
            if (g == 0) {
                int ws = 0;
                for (int z = 0; z < 32; z++) ws += wb[z];
                sum += -128 * ws;
            }
            acc[lane] = fmaf((float)sum, wd[b] * xd[b], acc[lane]);
        }
    return reduce16(acc);
}
/* gemma2_fast_x86.c:66-103 (q8_tile_vnni512, waves of at most 8 tokens):
 * 8 fp32 lanes per output, lane g taking the int32 sum of bytes 4g..4g+3 of
 * each block, float(sum) * (dw * dx) fused into the lane, then hsum8. */
static float q8_dot_vnni256(const int8_t *w, const int8_t *x, const float *wd, const float *xd, int kb) {
    float acc[8] = {0};
    for (int b = 0; b < kb; b++)
        for (int g = 0; g < 8; g++) {
            int sum = 0;
            for (int i = 4 * g; i < 4 * g + 4; i++) sum += w[(size_t)b * 32 + i] * x[(size_t)b * 32 + i];
            acc[g] = fmaf((float)sum, wd[b] * xd[b], acc[g]);
        }
    return hsum8(acc);
}
static void gemm_q8_rows(void *c, int t0, int t1) {
    const gemm_q8_job *j = c;
    int kb = j->k / 32;
    if (order_vnni) {
        for (int t = t0; t < t1; t++)
            for (int r = 0; r < j->m; r++) {
                const int8_t *w = j->wq + (size_t)r * j->k, *x = j->xq + (size_t)t * j->k;
                const float *wd = j->wd + (size_t)r * kb, *xd = j->xd + (size_t)t * kb;
                j->y[(size_t)t * j->m + r] = j->n > 8 && kb % 2 == 0 ? q8_dot_vnni512(w, x, wd, xd, kb)
                                                                     : q8_dot_vnni256(w, x, wd, xd, kb);
            }
        return;
    }
    for (int t = t0; t < t1; t++)
        for (int r = 0; r < j->m; r++) {
            float sum = 0;
            for (int i = 0; i < kb; i++) {
                const int p = variant_gemm_descending ? kb - 1 - i : i;
                const int8_t *a = j->wq + ((size_t)r * kb + p) * 32, *b = j->xq + ((size_t)t * kb + p) * 32;
                int dot = 0;
                for (int z = 0; z < 32; z++) dot += a[z] * b[z];
                sum += (float)dot * j->wd[(size_t)r * kb + p] * j->xd[(size_t)t * kb + p];
            }
            j->y[(size_t)t * j->m + r] = sum;
        }
}
static float *widen_fp16(const uint16_t *h, size_t count) {
    float *f = malloc(count * sizeof(float));
    for (size_t i = 0; i < count; i++) f[i] = eg2o_fp16_to_fp32(h[i]);
    return f;
}
void eg2o_gemm_q8(const int8_t *wq, const uint16_t *wd, const int8_t *xq, const uint16_t *xd,
                  int n, int k, int m, float *y) {
    float *wf = widen_fp16(wd, (size_t)m * (k / 32)), *xf = widen_fp16(xd, (size_t)n * (k / 32));
    gemm_q8_job j = {wq, xq, wf, xf, k, m, y, NULL, n};
    par_for(n, gemm_q8_rows, &j);
    free(wf), free(xf);
}

static void blockdot_rows(void *c, int t0, int t1) {
    const gemm_q8_job *j = c;
    int kb = j->k / 32;
    for (int t = t0; t < t1; t++)
        for (int r = 0; r < j->m; r++)
            for (int p = 0; p < kb; p++) {
                const int8_t *a = j->wq + ((size_t)r * kb + p) * 32, *b = j->xq + ((size_t)t * kb + p) * 32;
                int dot = 0;
                for (int z = 0; z < 32; z++) dot += a[z] * b[z];
                j->D[((size_t)t * j->m + r) * kb + p] = dot;
            }
}
void eg2o_gemm_q8_blockdots(const int8_t *wq, const int8_t *xq, int n, int k, int m, int32_t *D) {
    gemm_q8_job j = {wq, xq, NULL, NULL, k, m, NULL, D, n};
    par_for(n, blockdot_rows, &j);
}

/* gemma2_fast.c:482-559 scalar branch -- float GEMM for the BF16 PLE projection. */
typedef struct {
    const uint16_t *w;
    const float *x;
    int n, k, m;
    float *y;
} gemm_bf16_job;
static void gemm_bf16_rows(void *c, int r0, int r1) {
    const gemm_bf16_job *j = c;
    float *row = malloc((size_t)j->k * sizeof(float));
    for (int r = r0; r < r1; r++) {
        for (int z = 0; z < j->k; z++) row[z] = bf16_to_fp32(j->w[(size_t)r * j->k + z]);
        for (int t = 0; t < j->n; t++) {
            const float *x = j->x + (size_t)t * j->k;
            float sum = 0;
            if (order_vnni) {
                /* g2x_dot4x4 (gemma2_fast_x86.c:260-279): 8 lanes of fused
                 * multiply-adds over z, then hsum8. */
                float acc[8] = {0};
                for (int z = 0; z < j->k; z += 8)
                    for (int i = 0; i < 8; i++) acc[i] = fmaf(row[z + i], x[z + i], acc[i]);
                sum = hsum8(acc);
            } else {
                for (int z = 0; z < j->k; z++) sum += row[z] * x[z];
            }
            j->y[(size_t)t * j->m + r] = sum;
        }
    }
    free(row);
}
void eg2o_gemm_bf16(const uint16_t *w, const float *x, int n, int k, int m, float *y) {
    gemm_bf16_job j = {w, x, n, k, m, y};
    par_for(m, gemm_bf16_rows, &j);
}

/* gemma2_fast.c:587-590 (scalar sum_squares) and :667-671 (rms_row). */
/* g2x_sum_squares (gemma2_fast_x86.c:280-289): two 8-lane accumulators over
 * 16-element chunks, fused multiply-adds, hsum8 of their sum. */
static float sum_squares_x86(const float *x, int d) {
    float s0[8] = {0}, s1[8] = {0}, v[8];
    int z = 0;
    for (; z + 16 <= d; z += 16)
        for (int i = 0; i < 8; i++) {
            s0[i] = fmaf(x[z + i], x[z + i], s0[i]);
            s1[i] = fmaf(x[z + 8 + i], x[z + 8 + i], s1[i]);
        }
    for (int i = 0; i < 8; i++) v[i] = s0[i] + s1[i];
    float s = hsum8(v);
    for (; z < d; z++) s += x[z] * x[z];
    return s;
}
void eg2o_rms_row(float *r, int d, const float *w) {
    float ss;
    if (order_vnni) {
        ss = sum_squares_x86(r, d);
    } else {
        double s = 0;
        for (int z = 0; z < d; z++) s += (double)r[z] * r[z];
        ss = (float)s;
    }
    float scale = 1.0f / sqrtf(ss / d + 1e-6f);
    for (int z = 0; z < d; z++) r[z] *= scale * (w ? w[z] : 1.0f);
}

/* gemma2_fast.c:116-129 -- theta = t * powf(base, -2z/d). */
void eg2o_rope_tables(int d, float *cos_out, float *sin_out) {
    float base = d == 512 ? 1000000.0f : 10000.0f;
    for (int t = 0; t < 8192; t++)
        for (int z = 0; z < d / 2; z++) {
            float theta = t * powf(base, -2.0f * z / d);
            cos_out[(size_t)t * d / 2 + z] = cosf(theta);
            sin_out[(size_t)t * d / 2 + z] = sinf(theta);
        }
}

static float *rope_cos[2], *rope_sin[2];
static void rope_init(void) {
    for (int b = 0; b < 2; b++) {
        int d = b ? 512 : 256;
        if (rope_cos[b]) continue;
        rope_cos[b] = malloc((size_t)8192 * d / 2 * 4);
        rope_sin[b] = malloc((size_t)8192 * d / 2 * 4);
        eg2o_rope_tables(d, rope_cos[b], rope_sin[b]);
    }
}

/* gemma2_fast.c:672-679. */
static void rope_row(float *r, int d, int pos) {
    int b = d == 512;
    const float *c = rope_cos[b] + (size_t)pos * d / 2, *s = rope_sin[b] + (size_t)pos * d / 2;
    for (int z = 0; z < d / 2; z++) {
        float a = r[z], bb = r[z + d / 2];
        r[z] = a * c[z] - bb * s[z];
        r[z + d / 2] = a * s[z] + bb * c[z];
    }
}

/* gemma2_fast.c:768-894 scalar branch.  Masked keys add exact zeros there, so
 * summing only the keys inside [lo, hi) in ascending order is identical. */
typedef struct {
    const float *q, *k, *v;
    const uint32_t *lo, *hi;
    int n, kv, d, window;
    float *a;
} attn_job;
static void attention_rows(void *c, int t0, int t1) {
    const attn_job *j = c;
    const int kv = j->kv, d = j->d, window = j->window;
    float *sc = malloc((size_t)j->n * sizeof(float));
    for (int t = t0; t < t1; t++)
        for (int hd = 0; hd < 4; hd++) {
            int kh = hd / (4 / kv), lo = (int)j->lo[t], hi = (int)j->hi[t];
            if (window) {
                if (t - window > lo) lo = t - window;
                if (t + window + 1 < hi) hi = t + window + 1;
            }
            const float *qr = j->q + ((size_t)t * 4 + hd) * d;
            float mx = -INFINITY, total = 0;
            for (int s = lo; s < hi; s++) {
                const float *kr = j->k + ((size_t)s * kv + kh) * d;
                float dot = 0;
                if (order_vnni) { /* g2x_dot4x4 (gemma2_fast.c:826-828) */
                    float acc[8] = {0};
                    for (int z = 0; z < d; z += 8)
                        for (int i = 0; i < 8; i++) acc[i] = fmaf(qr[z + i], kr[z + i], acc[i]);
                    dot = hsum8(acc);
                } else {
                    for (int z = 0; z < d; z++) dot += qr[z] * kr[z];
                }
                sc[s] = dot;
                if (dot > mx) mx = dot;
            }
            for (int s = lo; s < hi; s++) {
                sc[s] = expf(sc[s] - mx);
                total += sc[s];
            }
            for (int s = lo; s < hi; s++) sc[s] /= total;
            float *o = j->a + ((size_t)t * 4 + hd) * d;
            /* g2x_pv (gemma2_fast_x86.c:326-349): one fused multiply-add per
             * key; the masked keys it also visits carry p = 0 and add +0. */
            for (int z = 0; z < d; z++) {
                float acc = 0;
                for (int s = lo; s < hi; s++)
                    acc = order_vnni ? fmaf(j->v[((size_t)s * kv + kh) * d + z], sc[s], acc)
                                     : acc + sc[s] * j->v[((size_t)s * kv + kh) * d + z];
                o[z] = acc;
            }
        }
    free(sc);
}
void eg2o_attention(const float *q, const float *k, const float *v, const uint32_t *lo_,
                    const uint32_t *hi_, int n, int kv, int d, int window, float *a) {
    attn_job j = {q, k, v, lo_, hi_, n, kv, d, window, a};
    par_for(n, attention_rows, &j);
}

/* AoS GGUF Q8_0 [rows][k] -> int8 plane + fp16 scale plane. */
static void unpack_q8(const void *src, int rows, int k, int8_t *q, uint16_t *d) {
    const uint8_t *b = src;
    for (size_t i = 0; i < (size_t)rows * k / 32; i++, b += 34) {
        memcpy(&d[i], b, 2);
        memcpy(q + i * 32, b + 2, 32);
    }
}

typedef struct {
    int8_t *q;
    uint16_t *d;
} q8w;
static q8w load_q8(const void *src, int rows, int k) {
    q8w w = {malloc((size_t)rows * k), malloc((size_t)rows * k / 32 * 2)};
    unpack_q8(src, rows, k, w.q, w.d);
    return w;
}
static void free_q8(q8w w) { free(w.q), free(w.d); }

/* gemm_q8 on a GGUF weight: unpack, then the scalar tile. */
static void gemm_w(const void *wt, int k, int m, const int8_t *xq, const uint16_t *xd, int n,
                   float *y) {
    q8w w = load_q8(wt, m, k);
    eg2o_gemm_q8(w.q, w.d, xq, xd, n, k, m, y);
    free_q8(w);
}

/* kernels.c:35-39,82-93,393-396 -- ei_l2_normalize with the SSE2 sum. */
static void l2_normalize_sse2(float *x, int n) {
    float s0[4] = {0}, s1[4] = {0};
    int i = 0;
    for (; i + 7 < n; i += 8)
        for (int j = 0; j < 4; j++) {
            s0[j] = s0[j] + x[i + j] * x[i + j];
            s1[j] = s1[j] + x[i + 4 + j] * x[i + 4 + j];
        }
    float v[4];
    for (int j = 0; j < 4; j++) v[j] = s0[j] + s1[j];
    float ss = (v[0] + v[2]) + (v[1] + v[3]);
    for (; i < n; i++) ss += x[i] * x[i];
    if (ss != 0.0f) {
        float sc = 1.0f / sqrtf(ss);
        for (int z = 0; z < n; z++) x[z] *= sc;
    }
}

#define T(i) (tensors[(i)])
#define LT(l, j) (tensors[3 + 17 * (l) + (j)])

/* Per-wave work buffers for up to `count` tokens. */
typedef struct {
    float *h, *q, *k, *v, *a, *up, *gate;
    int8_t *xq;
    uint16_t *xd;
    uint32_t *lo, *hi, *pos;
} wave_ws;

static wave_ws ws_alloc(const size_t *offsets, size_t batch) {
    size_t count = offsets[batch];
    wave_ws w = {malloc(count * 512 * 4), malloc(count * 2048 * 4), malloc(count * 512 * 4), malloc(count * 512 * 4),
                 malloc(count * 2048 * 4), malloc(count * 2048 * 4), malloc(count * 2048 * 4),
                 malloc(count * 2048), malloc(count * 64 * 2),
                 malloc(count * 4), malloc(count * 4), malloc(count * 4)};
    for (size_t s = 0; s < batch; s++)
        for (size_t t = offsets[s]; t < offsets[s + 1]; t++)
            w.lo[t] = (uint32_t)offsets[s], w.hi[t] = (uint32_t)offsets[s + 1], w.pos[t] = (uint32_t)(t - offsets[s]);
    return w;
}
static void ws_free(wave_ws *w) {
    free(w->h), free(w->q), free(w->k), free(w->v), free(w->a), free(w->up), free(w->gate);
    free(w->xq), free(w->xd), free(w->lo), free(w->hi), free(w->pos);
}

/* gemma2_fast.c:951-956 -- ple = rms(x . W_ple^T / sqrt(512)) per 512-slice. */
static void ple_project(const void *const *tensors, const float *x, int n, float *ple) {
    size_t count = (size_t)n;
    eg2o_gemm_bf16(T(1), x, n, 512, 24 * 512, ple);
    for (size_t i = 0; i < count * 512 * 24; i++) ple[i] /= sqrtf(512.0f);
    for (size_t r = 0; r < count * 24; r++) eg2o_rms_row(ple + r * 512, 512, T(2));
}

/* One layer of the loop at gemma2_fast.c:957-992, x updated in place. */
static void layer_forward(const void *const *tensors, int l, float *x, const float *ple, int n, int qm, int gm,
                          wave_ws *w) {
    int d = l % 6 == 5 ? 512 : 256, kv = 512 / d;
    float *h = w->h, *q = w->q, *k = w->k, *v = w->v, *a = w->a, *up = w->up, *gate = w->gate;
    int8_t *xq = w->xq;
    uint16_t *xd = w->xd;
    /* ROW_NORM_QUANT (gemma2_fast.c:685-691). */
    for (int t = 0; t < n; t++) {
        memcpy(h + (size_t)t * 512, x + (size_t)t * 512, 2048);
        eg2o_rms_row(h + (size_t)t * 512, 512, LT(l, 0));
    }
    eg2o_quantize(h, xq, xd, n * 512, qm);
    gemm_w(LT(l, 1), 512, 4 * d, xq, xd, n, q);
    gemm_w(LT(l, 2), 512, 512, xq, xd, n, k);
    gemm_w(LT(l, 3), 512, 512, xq, xd, n, v);
    /* ROW_QKV_POST (gemma2_fast.c:692-706). */
    for (int t = 0; t < n; t++) {
        for (int hd = 0; hd < 4; hd++) {
            float *r = q + ((size_t)t * 4 + hd) * d;
            eg2o_rms_row(r, d, LT(l, 5));
            rope_row(r, d, (int)w->pos[t]);
        }
        for (int hd = 0; hd < kv; hd++) {
            float *r = k + ((size_t)t * kv + hd) * d;
            eg2o_rms_row(r, d, LT(l, 6));
            rope_row(r, d, (int)w->pos[t]);
            eg2o_rms_row(v + ((size_t)t * kv + hd) * d, d, NULL);
        }
    }
    if (variant_attention_fp16) {
        for (size_t i = 0; i < (size_t)n * 4 * d; i++) q[i] = (float)(_Float16)q[i];
        for (size_t i = 0; i < (size_t)n * kv * d; i++) k[i] = (float)(_Float16)k[i], v[i] = (float)(_Float16)v[i];
    }
    eg2o_attention(q, k, v, w->lo, w->hi, n, kv, d, l % 6 == 5 ? 0 : 512, a);
    /* ROW_QUANT(a) -> attn_output -> ROW_POST_ADD (gemma2_fast.c:972-975). */
    eg2o_quantize(a, xq, xd, n * 4 * d, qm);
    gemm_w(LT(l, 4), 4 * d, 512, xq, xd, n, h);
    for (int t = 0; t < n; t++) {
        float *hh = h + (size_t)t * 512, *xx = x + (size_t)t * 512;
        eg2o_rms_row(hh, 512, LT(l, 7));
        for (int z = 0; z < 512; z++) xx[z] = (xx[z] + hh[z]) * 1.0f;
    }
    /* FFN (gemma2_fast.c:976-983). */
    for (int t = 0; t < n; t++) {
        memcpy(h + (size_t)t * 512, x + (size_t)t * 512, 2048);
        eg2o_rms_row(h + (size_t)t * 512, 512, LT(l, 8));
    }
    eg2o_quantize(h, xq, xd, n * 512, qm);
    gemm_w(LT(l, 9), 512, 2048, xq, xd, n, up);
    gemm_w(LT(l, 10), 512, 2048, xq, xd, n, gate);
    eg2o_gelu_mul(gate, up, n * 2048, gm);
    eg2o_quantize(gate, xq, xd, n * 2048, qm);
    gemm_w(LT(l, 11), 2048, 512, xq, xd, n, h);
    for (int t = 0; t < n; t++) {
        float *hh = h + (size_t)t * 512, *xx = x + (size_t)t * 512;
        eg2o_rms_row(hh, 512, LT(l, 12));
        for (int z = 0; z < 512; z++) xx[z] = (xx[z] + hh[z]) * 1.0f;
    }
    /* Per-layer embedding gate (gemma2_fast.c:984-990). */
    eg2o_quantize(x, xq, xd, n * 512, qm);
    gemm_w(LT(l, 13), 512, 512, xq, xd, n, h);
    for (int t = 0; t < n; t++)
        eg2o_gelu_mul(h + (size_t)t * 512, ple + ((size_t)t * 24 + l) * 512, 512, gm);
    eg2o_quantize(h, xq, xd, n * 512, qm);
    gemm_w(LT(l, 14), 512, 512, xq, xd, n, a);
    float scale = *(const float *)LT(l, 16);
    for (int t = 0; t < n; t++) {
        float *hh = a + (size_t)t * 512, *xx = x + (size_t)t * 512;
        eg2o_rms_row(hh, 512, LT(l, 15));
        for (int z = 0; z < 512; z++) xx[z] = (xx[z] + hh[z]) * scale;
    }
}

static int embed_batch(const void *const *tensors, const int32_t *ids, const float *inputs,
                       const size_t *offsets, size_t batch, float *out, int qm, int gm, float *x_layers,
                       float *ple_out);

int eg2o_embed_batch(const void *const *tensors, const int32_t *ids, const size_t *offsets,
                     size_t batch, float *out, int qm, int gm, float *x_layers) {
    return embed_batch(tensors, ids, NULL, offsets, batch, out, qm, gm, x_layers, NULL);
}

int eg2o_embed_trace(const void *const *tensors, const int32_t *ids, const size_t *offsets, size_t batch,
                     float *out, int qm, int gm, float *x_layers, float *ple_out) {
    return embed_batch(tensors, ids, NULL, offsets, batch, out, qm, gm, x_layers, ple_out);
}

/* gemma2_fast.c:940-941: with ids NULL the wave starts from caller-given
 * 512-wide rows (media soft tokens), copied into x unscaled. */
int eg2o_embed_batch_inputs(const void *const *tensors, const float *inputs, const size_t *offsets,
                            size_t batch, float *out, int qm, int gm) {
    return inputs ? embed_batch(tensors, NULL, inputs, offsets, batch, out, qm, gm, NULL, NULL) : 1;
}

int eg2o_layer(const void *const *tensors, int l, float *x, const float *ple, const size_t *offsets, size_t batch,
               int qm, int gm) {
    size_t count = offsets[batch];
    if (!count || count > 8192 || l < 0 || l >= 24) return 1;
    rope_init();
    wave_ws w = ws_alloc(offsets, batch);
    layer_forward(tensors, l, x, ple, (int)count, qm, gm, &w);
    ws_free(&w);
    return 0;
}

static int embed_batch(const void *const *tensors, const int32_t *ids, const float *inputs,
                       const size_t *offsets, size_t batch, float *out, int qm, int gm, float *x_layers,
                       float *ple_out) {
    size_t count = offsets[batch];
    if (!count || count > 8192) return 1;
    int n = (int)count;
    rope_init();
    float *x = malloc(count * 512 * 4);
    float *ple = ple_out ? ple_out : malloc(count * 512 * 24 * 4);
    wave_ws w = ws_alloc(offsets, batch);
    /* gemma2_fast.c:940-950: x = the given rows, or (d * q) * sqrtf(512). */
    if (inputs) memcpy(x, inputs, count * 512 * 4);
    for (int t = 0; t < n && !inputs; t++) {
        const uint8_t *row = (const uint8_t *)T(0) + (size_t)ids[t] * 16 * 34;
        for (int b = 0; b < 16; b++) {
            uint16_t hb;
            memcpy(&hb, row + b * 34, 2);
            float d = eg2o_fp16_to_fp32(hb);
            const int8_t *qs = (const int8_t *)(row + b * 34 + 2);
            for (int z = 0; z < 32; z++) x[(size_t)t * 512 + b * 32 + z] = d * qs[z] * sqrtf(512.0f);
        }
    }
    ple_project(tensors, x, n, ple);
    for (int l = 0; l < 24; l++) {
        if (x_layers) memcpy(x_layers + (size_t)l * count * 512, x, count * 512 * 4);
        layer_forward(tensors, l, x, ple, n, qm, gm, &w);
    }
    if (x_layers) memcpy(x_layers + (size_t)24 * count * 512, x, count * 512 * 4);
    /* Output head and pooling (gemma2_fast.c:993-1008). */
    float *h = w.h;
    int8_t *xq = w.xq;
    uint16_t *xd = w.xd;
    for (int t = 0; t < n; t++) {
        memcpy(h + (size_t)t * 512, x + (size_t)t * 512, 2048);
        eg2o_rms_row(h + (size_t)t * 512, 512, T(3 + 17 * 24));
    }
    eg2o_quantize(h, xq, xd, n * 512, qm);
    float *y = malloc(count * 768 * 4);
    gemm_w(T(4 + 17 * 24), 512, 768, xq, xd, n, y);
    for (size_t s = 0; s < batch; s++) {
        float *o = out + s * 768;
        size_t len = offsets[s + 1] - offsets[s];
        memset(o, 0, 768 * 4);
        for (size_t t = offsets[s]; t < offsets[s + 1]; t++)
            for (int z = 0; z < 768; z++) o[z] += y[t * 768 + z] / (float)len;
        l2_normalize_sse2(o, 768);
    }
    free(y), free(x);
    if (!ple_out) free(ple);
    ws_free(&w);
    return 0;
}
