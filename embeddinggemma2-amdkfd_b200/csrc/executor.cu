// EmbeddingGemma 2 packed-wave executor for B200: the C ABI of
// include/eg2_executor.h, replacing src/gemma2_kfd.cpp of the reference.
//
// Structure (reference -> here):
//   KFD context, queue, code object (gemma2_kfd.cpp:86-155)
//       -> one CUDA stream per context on a chosen device, kernel attributes;
//   GGUF bytes copied to GTT, arena for 2048 tokens (:111-115)
//       -> Q8_0 weights repacked once into int8 code planes + fp32 block-scale
//          planes (TMA-friendly rows), q/k/v fused into one projection per
//          layer; token_embd kept as GGUF blocks for the gather; device arena
//          sized for 2048 packed tokens;
//   PM4/AQL command buffers with a wait after every dispatch and chunked
//   flushes (:156-225) -> one CUDA graph per wave shape (tokens, sequences),
//          captured on first use and replayed;
//   host bounds / RoPE tables (:286-296) -> per-token bounds and positions
//          uploaded per wave; RoPE tables built once with the reference CPU
//          graph's expression (gemma2_fast.c:116-129);
//   30 s submit/wait timeout and poisoning (:21,190-214) -> a deadline while
//          polling the wave's completion event, plus the device error word set
//          by bounded in-kernel waits; either poisons the context.
#include <atomic>
#include <chrono>
#include <cmath>
#include <condition_variable>
#include <exception>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "../../include/eg2_executor.h"
#include "../../include/gemma2_cuda.h"
#include "launch.h"

namespace {
using namespace eg2;

constexpr unsigned CAP = 2048;  // packed tokens per wave: the reference's KFD cap (gemma2_kfd.cpp:20)
// EG2_B200_WAVE_8192: the reference CPU graph's wave limit (gemma2_fast.c:924-925).
constexpr unsigned WIDE_CAP = 8192;
// Waves run padded to a multiple of BUCKET tokens: the padding is one extra
// sequence that the pooling skips, and every kernel is per token or per
// sequence, so the real tokens' results do not change.  One CUDA graph per
// bucket then serves every wave shape (at most cap / BUCKET graphs).
constexpr unsigned BUCKET = 64;
constexpr int VOCAB = 262144;
constexpr double TIMEOUT_S = 30.0;  // gemma2_kfd.cpp:21

void ck(cudaError_t e, const char *what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// The token-count message: the KFD executor's (gemma2_kfd.cpp:271) at its cap,
// the CPU graph's (gemma2_fast.c:925) for 8192-token waves.
const char *count_message(unsigned cap) {
    return cap > CAP ? "EmbeddingGemma 2 accepts 1..8192 input tokens"
                     : "KFD batch requires 1..2048 packed tokens and nonempty sequences";
}

// gemma2_kfd.cpp:270-278: the same checks, in the same order, with its messages.
void validate_wave(const int32_t *ids, const size_t *offsets, size_t batch, unsigned cap = CAP) {
    if (!ids || !offsets || !batch || batch > cap || offsets[0] || offsets[batch] > cap)
        throw std::runtime_error(count_message(cap));
    for (size_t s = 0; s < batch; ++s)
        if (offsets[s + 1] <= offsets[s]) throw std::runtime_error("invalid KFD sequence offsets");
    const size_t n = offsets[batch];
    for (size_t i = 0; i < n; ++i)
        if (ids[i] < 0 || ids[i] >= VOCAB) throw std::runtime_error("token ID out of range");
}

// Media soft-token waves (ids NULL, 512-wide input rows: gemma2_fast.c:940-941)
// take the same offsets checks and messages; the rows themselves are not
// inspected, as in the reference.
void validate_rows(const float *rows, const size_t *offsets, size_t batch, unsigned cap = CAP) {
    if (!rows || !offsets || !batch || batch > cap || offsets[0] || offsets[batch] > cap)
        throw std::runtime_error(count_message(cap));
    for (size_t s = 0; s < batch; ++s)
        if (offsets[s + 1] <= offsets[s]) throw std::runtime_error("invalid KFD sequence offsets");
}

struct Q8Weight {
    int8_t *codes = nullptr;  // [rows][k]
    float *scales = nullptr;  // [k/32][rows]
    int rows = 0, k = 0;
    CUtensorMap tmap{}, tscale{};
};

struct Layer {
    int d = 256, kv = 2;
    Q8Weight qkv, o, gu, down, inp_gate, proj;  // gu: gate/up interleaved in 64-row chunks
    const float *attn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr, *post_attn_norm = nullptr,
                *ffn_norm = nullptr, *post_ffw_norm = nullptr, *post_norm = nullptr, *out_scale = nullptr;
};

struct Profiler {
    cudaStream_t s;
    std::vector<std::string> names;
    std::vector<cudaEvent_t> events;
    void mark(const char *name) {
        cudaEvent_t e;
        ck(cudaEventCreate(&e), "cudaEventCreate");
        events.push_back(e);
        names.emplace_back(name);
        ck(cudaEventRecord(e, s), "cudaEventRecord");
    }
    ~Profiler() {
        for (auto e : events) cudaEventDestroy(e);
    }
};

// One wave's device working set: its stream, the per-wave input block, the
// activation arena for cap packed tokens, the tensor maps over it, the CUDA
// graphs captured against it, and the pinned host staging of the pipeline slot
// that runs on it.  A context holds LANES of them over one set of weights, so
// two submitted waves run concurrently on the GPU (each wave's ~300 kernels
// leave SMs idle in their ramps and tails, which the other wave's kernels fill).
struct Lane {
    cudaStream_t stream = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;  // launch(): lane 0 -> this lane -> lane 0
    int *ids = nullptr;
    unsigned *bounds = nullptr, *pos = nullptr, *offsets = nullptr, *seq_count = nullptr;
    float *xin = nullptr;  // soft-token waves: the uploaded input rows [cap][512]
    float *x = nullptr, *ple = nullptr, *qkv = nullptr, *attn = nullptr, *h = nullptr, *y = nullptr, *pooled = nullptr,
          *xs = nullptr, *gs = nullptr;
    void *x_hi = nullptr, *x_lo = nullptr, *qh = nullptr, *kh = nullptr, *vh = nullptr;
    int8_t *xq = nullptr, *gq = nullptr;  // Q8 activations; gq/gs: the GeGLU output (FFN down operand)
    float *qf = nullptr, *kf = nullptr, *vf = nullptr;  // parity mode: fp32 q/k/v
    CUtensorMap tm_xq[3]{}, tm_xs[3]{}, tm_gq{}, tm_gs{}, tm_hi{}, tm_lo{};
    std::map<uint64_t, cudaGraphExec_t> graphs;  // per wave shape
    cudaGraphExec_t staged_graph = nullptr;
    // Host staging (pinned) of the pipeline slot on this lane.
    uint32_t *in = nullptr;  // ids | bounds(2) | pos | offsets | sequence count
    float *rows = nullptr;   // soft-token waves: [cap][512] input rows (allocated on first use)
    float *out = nullptr;
    int *err = nullptr;  // the device error word, read back with the wave
    cudaEvent_t done = nullptr;
    size_t batch = 0;
    bool busy = false;     // a wave on this lane is not delivered yet
    bool by_call = false;  // ... and a synchronous call (not submit) owns it
};

struct Backend {
    const ei_gguf *model;
    int device = 0;
    cudaStream_t stream = nullptr;  // weight upload; then the first lane's stream
    std::mutex mutex;
    std::condition_variable lane_freed;  // a synchronous call released its lane
    std::atomic<bool> poisoned{false};

    std::vector<void *> allocations;
    std::vector<Layer> layers;
    Q8Weight output;
    const uint8_t *token_embd = nullptr;
    const void *ple_w = nullptr;
    const float *ple_norm = nullptr, *output_norm = nullptr;
    float *rope_cos[2] = {}, *rope_sin[2] = {};

    CUtensorMap tm_ple{};
    // Parity mode (EG2_B200_EXACT): GEMMs in the reference scalar tile's rounding
    // order, PLE projection and attention on the CUDA-core exact-order kernels
    // with fp32 q/k/v; every other kernel is bit-exact in both modes.
    bool exact = false;
    // Packed tokens per wave: CAP, or WIDE_CAP with EG2_B200_WAVE_8192.
    unsigned cap = CAP;
    // EG2_B200_SCALAR_TIER: the scalar CPU tier's quantizer rounding and GELU
    // (roundf, tanhf) instead of the x86 tiers' (the fast path's choice).
    int tier = 0;

    // Pipeline slot i runs on lane i: a wave can be submitted to one slot
    // while the other slot's wave is still on the GPU, on its own stream and
    // arena.
    static constexpr int LANES = 2;
    Lane lanes[LANES];
    int next_slot = 0;

    // The split form's staged wave (the same inputs staged in every lane).
    unsigned staged_n = 0;
    bool staged_rows = false, staged = false;
    size_t staged_batch = 0;
    int kernels_per_wave = 0;

    template <class T>
    T *dalloc(size_t count) {
        void *p = nullptr;
        ck(cudaMalloc(&p, count * sizeof(T) + 256), "cudaMalloc");
        allocations.push_back(p);
        return static_cast<T *>(p);
    }

    const ei_tensor *tensor(const std::string &name) const {
        for (uint64_t i = 0; i < model->n_tensors; i++) {
            const ei_tensor &t = model->tensors[i];
            if (t.name.len == name.size() && !std::memcmp(t.name.str, name.data(), t.name.len)) return &t;
        }
        throw std::runtime_error("missing tensor: " + name);
    }
    void check_shape(const ei_tensor *t, uint64_t k, uint64_t m, uint32_t type, const std::string &name) const {
        if (t->ne[0] != k || t->ne[1] != m || t->ne[2] != 1 || t->ne[3] != 1 || t->type != type)
            throw std::runtime_error("unsupported tensor " + name);
    }
    uint64_t kv_u64(const char *key) const {
        for (uint64_t i = 0; i < model->n_kv; i++) {
            const ei_kv &kv = model->kv[i];
            if (kv.key.len == std::strlen(key) && !std::memcmp(kv.key.str, key, kv.key.len)) return kv.v.u64;
        }
        return 0;
    }

    // f32 norm weight -> device (tensor must be F32, as gemma2_kfd.cpp:81-85 requires).
    const float *norm_weight(const std::string &name, uint64_t len, float *&cursor) {
        const ei_tensor *t = tensor(name);
        check_shape(t, len, 1, 0, name);
        float *dst = cursor;
        ck(cudaMemcpy(dst, t->data, len * 4, cudaMemcpyHostToDevice), "norm upload");
        cursor += (len + 63) / 64 * 64;
        return dst;
    }

    // GGUF Q8_0 [rows][k] -> SoA planes at row offset `row0` of a fused weight.
    void repack(const std::string &name, int k, int rows, Q8Weight &w, int row0, uint8_t *staging) {
        const ei_tensor *t = tensor(name);
        check_shape(t, uint64_t(k), uint64_t(rows), 8, name);
        ck(cudaMemcpyAsync(staging, t->data, t->n_bytes, cudaMemcpyHostToDevice, stream), "weight upload");
        ck(launch_repack_q8(staging, rows, k, w.codes + size_t(row0) * k, w.scales + row0, w.rows, stream), "repack");
        ck(cudaStreamSynchronize(stream), "repack sync");  // staging is reused by the next tensor
    }
    // Gate and up matrices [rows][k] into one weight interleaved in 64-row chunks
    // (the fused GeGLU GEMM's layout): rows 128c.. = gate rows 64c.., rows
    // 128c+64.. = up rows 64c...
    void repack_geglu(const std::string &gate, const std::string &up, int k, int rows, Q8Weight &w,
                      uint8_t *staging) {
        for (int half = 0; half < 2; ++half) {
            const ei_tensor *t = tensor(half ? up : gate);
            check_shape(t, uint64_t(k), uint64_t(rows), 8, half ? up : gate);
            ck(cudaMemcpyAsync(staging, t->data, t->n_bytes, cudaMemcpyHostToDevice, stream), "weight upload");
            ck(launch_repack_q8(staging, rows, k, w.codes, w.scales, w.rows, stream, 64, half), "repack");
            ck(cudaStreamSynchronize(stream), "repack sync");
        }
    }
    void alloc_q8(Q8Weight &w, int rows, int k) {
        w.rows = rows, w.k = k;
        w.codes = dalloc<int8_t>(size_t(rows) * k);
        w.scales = dalloc<float>(size_t(rows) * (k / 32));
    }
    void finish_q8(Q8Weight &w) {
        if (w.rows % 128 || !q8_tmap(&w.tmap, w.codes, uint64_t(w.k), uint64_t(w.rows), 128) ||
            !scale_tmap(&w.tscale, w.scales, uint64_t(w.rows), uint64_t(w.k / 32), 128))
            throw std::runtime_error("cuTensorMapEncodeTiled failed for a weight");
    }

    Backend(const ei_gguf *g, int dev, unsigned flags)
        : model(g), device(dev), exact(flags & EG2_B200_EXACT), cap(flags & EG2_B200_WAVE_8192 ? WIDE_CAP : CAP),
          tier(flags & EG2_B200_SCALAR_TIER ? TIER_SCALAR : flags & EG2_B200_VNNI512_TIER ? TIER_VNNI512 : TIER_X86) {
        if (!g) throw std::runtime_error("empty model");
        if ((flags & EG2_B200_VNNI512_TIER) && (!exact || (flags & EG2_B200_SCALAR_TIER)))
            throw std::runtime_error("EG2_B200_VNNI512_TIER needs EG2_B200_EXACT and excludes EG2_B200_SCALAR_TIER");
        // The exact-order attention keeps a row's scores in shared memory.
        if (exact && cap > CAP) throw std::runtime_error("parity mode supports waves of up to 2048 tokens");
        // gemma2.c:30-62 hyperparameters.
        if (kv_u64("gemma-embedding2.block_count") != 24 || kv_u64("gemma-embedding2.embedding_length") != 512 ||
            kv_u64("gemma-embedding2.feed_forward_length") != 2048 ||
            kv_u64("gemma-embedding2.embedding_length_out") != 768 ||
            kv_u64("gemma-embedding2.attention.sliding_window") != 1024)
            throw std::runtime_error("unsupported EmbeddingGemma 2 hyperparameters");
        int count = 0;
        ck(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
        if (device < 0 || device >= count)
            throw std::runtime_error("CUDA device " + std::to_string(device) + " not found");
        ck(cudaSetDevice(device), "cudaSetDevice");
        cudaDeviceProp prop;
        ck(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
        if (prop.major != 10 || prop.minor != 0)
            throw std::runtime_error(std::string("supported CUDA device not found (sm_100 required, got ") +
                                     prop.name + ")");
        for (Lane &ln : lanes) {
            ck(cudaStreamCreateWithFlags(&ln.stream, cudaStreamNonBlocking), "cudaStreamCreate");
            for (cudaEvent_t *e : {&ln.done, &ln.fork, &ln.join})
                ck(cudaEventCreateWithFlags(e, cudaEventDisableTiming), "cudaEventCreate");
        }
        stream = lanes[0].stream;
        ck(init_kernel_attributes(), "kernel attributes");

        // ---- weights
        const ei_tensor *emb = tensor("token_embd.weight");
        check_shape(emb, 512, VOCAB, 8, "token_embd.weight");
        auto *emb_d = dalloc<uint8_t>(emb->n_bytes);
        ck(cudaMemcpy(emb_d, emb->data, emb->n_bytes, cudaMemcpyHostToDevice), "token_embd upload");
        token_embd = emb_d;
        const ei_tensor *plew = tensor("per_layer_model_proj.weight");
        check_shape(plew, 512, 24 * 512, 30, "per_layer_model_proj.weight");
        auto *ple_d = dalloc<uint8_t>(plew->n_bytes);
        ck(cudaMemcpy(ple_d, plew->data, plew->n_bytes, cudaMemcpyHostToDevice), "PLE upload");
        ple_w = ple_d;

        float *norms = dalloc<float>(size_t(256) * 1024);
        float *cur = norms;
        ple_norm = norm_weight("per_layer_proj_norm.weight", 512, cur);
        output_norm = norm_weight("output_norm.weight", 512, cur);
        uint8_t *staging = dalloc<uint8_t>(size_t(2048) * 2048 / 32 * 34);
        layers.resize(24);
        for (int l = 0; l < 24; ++l) {
            Layer &L = layers[l];
            L.d = l % 6 == 5 ? 512 : 256, L.kv = 512 / L.d;
            const std::string p = "blk." + std::to_string(l) + ".";
            auto nm = [&](const char *s) { return p + s + ".weight"; };
            L.attn_norm = norm_weight(nm("attn_norm"), 512, cur);
            L.q_norm = norm_weight(nm("attn_q_norm"), L.d, cur);
            L.k_norm = norm_weight(nm("attn_k_norm"), L.d, cur);
            L.post_attn_norm = norm_weight(nm("post_attention_norm"), 512, cur);
            L.ffn_norm = norm_weight(nm("ffn_norm"), 512, cur);
            L.post_ffw_norm = norm_weight(nm("post_ffw_norm"), 512, cur);
            L.post_norm = norm_weight(nm("post_norm"), 512, cur);
            L.out_scale = norm_weight(nm("layer_output_scale"), 1, cur);
            alloc_q8(L.qkv, 4 * L.d + 1024, 512);
            repack(nm("attn_q"), 512, 4 * L.d, L.qkv, 0, staging);
            repack(nm("attn_k"), 512, 512, L.qkv, 4 * L.d, staging);
            repack(nm("attn_v"), 512, 512, L.qkv, 4 * L.d + 512, staging);
            alloc_q8(L.o, 512, 4 * L.d);
            repack(nm("attn_output"), 4 * L.d, 512, L.o, 0, staging);
            alloc_q8(L.gu, 4096, 512);
            repack_geglu(nm("ffn_gate"), nm("ffn_up"), 512, 2048, L.gu, staging);
            alloc_q8(L.down, 512, 2048);
            repack(nm("ffn_down"), 2048, 512, L.down, 0, staging);
            alloc_q8(L.inp_gate, 512, 512);
            repack(nm("inp_gate"), 512, 512, L.inp_gate, 0, staging);
            alloc_q8(L.proj, 512, 512);
            repack(nm("proj"), 512, 512, L.proj, 0, staging);
            for (Q8Weight *w : {&L.qkv, &L.o, &L.gu, &L.down, &L.inp_gate, &L.proj}) finish_q8(*w);
        }
        alloc_q8(output, 768, 512);
        repack("output.weight", 512, 768, output, 0, staging);
        finish_q8(output);

        // ---- RoPE tables for in-sequence positions 0..cap-1 (gemma2_fast.c:116-129)
        for (int b = 0; b < 2; ++b) {
            const int d = b ? 512 : 256;
            const float base = b ? 1000000.0f : 10000.0f;
            std::vector<float> c(size_t(cap) * d / 2), s(size_t(cap) * d / 2);
            for (unsigned t = 0; t < cap; ++t)
                for (int z = 0; z < d / 2; ++z) {
                    const float theta = float(t) * powf(base, -2.0f * float(z) / float(d));
                    c[size_t(t) * d / 2 + z] = cosf(theta);
                    s[size_t(t) * d / 2 + z] = sinf(theta);
                }
            rope_cos[b] = dalloc<float>(c.size());
            rope_sin[b] = dalloc<float>(s.size());
            ck(cudaMemcpy(rope_cos[b], c.data(), c.size() * 4, cudaMemcpyHostToDevice), "rope upload");
            ck(cudaMemcpy(rope_sin[b], s.data(), s.size() * 4, cudaMemcpyHostToDevice), "rope upload");
        }

        if (!bf16_tmap(&tm_ple, ple_w, 512, 24 * 512, 256)) throw std::runtime_error("tensor map (PLE)");
        for (Lane &ln : lanes) alloc_lane(ln);
        ck(cudaStreamSynchronize(stream), "weight upload");
        // The device error word is not cleared here: it is shared by every
        // context on this device, and a wave of another context may have set it
        // a moment ago (it would then go unreported).  A set word fails the
        // next wave of every context on the device, this one included.
        // EG2_B200_PREPARE_TOKENS=n: capture every wave shape up to n tokens
        // now, so that no request pays a graph capture (for callers that
        // cannot call eg2_b200_prepare, e.g. the reference's server).
        if (const char *prep = std::getenv("EG2_B200_PREPARE_TOKENS")) prepare(unsigned(std::atoi(prep)));
        if (std::getenv("EG2_B200_VERBOSE")) {
            size_t free_b = 0, total_b = 0;
            cudaMemGetInfo(&free_b, &total_b);
            std::fprintf(stderr, "B200: device %d (%s), %zu allocations, %.1f MiB free, cap %u packed tokens\n", device,
                         prop.name, allocations.size(), free_b / 1048576.0, cap);
        }
    }

    // The arena of one lane for cap packed tokens.  The per-wave inputs share
    // one block laid out like the pinned staging buffer (ids | bounds | pos |
    // offsets | count), so a wave uploads them with a single copy.
    void alloc_lane(Lane &ln) {
        unsigned *in_block = dalloc<unsigned>(5 * cap + 2);
        ln.ids = reinterpret_cast<int *>(in_block);
        ln.bounds = in_block + cap;
        ln.pos = in_block + 3 * cap;
        ln.offsets = in_block + 4 * cap;
        ln.seq_count = in_block + 5 * cap + 1;
        ln.x = dalloc<float>(size_t(cap) * 512);
        ln.x_hi = dalloc<uint16_t>(size_t(cap) * 512);
        ln.x_lo = dalloc<uint16_t>(size_t(cap) * 512);
        ln.ple = dalloc<float>(size_t(cap) * 24 * 512);
        ln.xq = dalloc<int8_t>(size_t(cap) * 2048);
        ln.xs = dalloc<float>(size_t(64) * cap);
        ln.qkv = dalloc<float>(size_t(cap) * 3072);
        ln.qh = dalloc<uint16_t>(size_t(cap) * 2048);
        ln.kh = dalloc<uint16_t>(size_t(cap) * 512);
        ln.vh = dalloc<uint16_t>(size_t(cap) * 512);
        ln.attn = dalloc<float>(size_t(cap) * 2048);
        ln.h = dalloc<float>(size_t(cap) * 512);
        ln.gq = dalloc<int8_t>(size_t(cap) * 2048);
        ln.gs = dalloc<float>(size_t(64) * cap);
        ln.y = dalloc<float>(size_t(cap) * 768);
        ln.pooled = dalloc<float>(size_t(cap) * 768);
        if (exact) {
            ln.qf = dalloc<float>(size_t(cap) * 2048);
            ln.kf = dalloc<float>(size_t(cap) * 512);
            ln.vf = dalloc<float>(size_t(cap) * 512);
        }
        const int ks[3] = {512, 1024, 2048};
        for (int i = 0; i < 3; ++i)
            if (!q8_tmap(&ln.tm_xq[i], ln.xq, uint64_t(ks[i]), cap, 64) ||
                !scale_tmap(&ln.tm_xs[i], ln.xs, cap, uint64_t(ks[i] / 32), 64))
                throw std::runtime_error("tensor map (activations)");
        if (!q8_tmap(&ln.tm_gq, ln.gq, 2048, cap, 64) || !scale_tmap(&ln.tm_gs, ln.gs, cap, 64, 64))
            throw std::runtime_error("tensor map (GeGLU activations)");
        if (!bf16_tmap(&ln.tm_hi, ln.x_hi, 512, cap, 128) || !bf16_tmap(&ln.tm_lo, ln.x_lo, 512, cap, 128))
            throw std::runtime_error("tensor map (PLE)");
        ck(cudaMallocHost(&ln.in, sizeof(uint32_t) * (5 * cap + 2)), "cudaMallocHost");
        ck(cudaMallocHost(&ln.err, sizeof(int)), "cudaMallocHost");
        ck(cudaMallocHost(&ln.out, sizeof(float) * cap * 768), "cudaMallocHost");
    }

    ~Backend() {
        if (device >= 0) cudaSetDevice(device);
        for (Lane &ln : lanes)
            if (ln.stream) cudaStreamSynchronize(ln.stream);
        for (Lane &ln : lanes)
            for (auto &kv : ln.graphs) cudaGraphExecDestroy(kv.second);
        for (void *p : allocations) cudaFree(p);
        for (Lane &ln : lanes) {
            if (ln.in) cudaFreeHost(ln.in);
            if (ln.rows) cudaFreeHost(ln.rows);
            if (ln.err) cudaFreeHost(ln.err);
            if (ln.out) cudaFreeHost(ln.out);
            for (cudaEvent_t e : {ln.done, ln.fork, ln.join})
                if (e) cudaEventDestroy(e);
            if (ln.stream) cudaStreamDestroy(ln.stream);
        }
    }

    static int kidx(int k) { return k == 512 ? 0 : k == 1024 ? 1 : 2; }
    // Parity mode at the VNNI-512 tier: the GEMMs in that tier's lane order.
    bool vnni() const { return exact && tier == TIER_VNNI512; }
    void gemm(const Lane &ln, const Q8Weight &w, float *out, int ldo, int n) {
        if (vnni())
            ck(launch_q8gemm_vnni(w.codes, w.scales, ln.xq, ln.xs, int(cap), out, nullptr, ldo, n, w.rows, w.k,
                                  ln.offsets, ln.seq_count, ln.stream),
               "q8 GEMM");
        else
            ck(launch_q8gemm(w.tmap, ln.tm_xq[kidx(w.k)], w.tscale, ln.tm_xs[kidx(w.k)], exact, out, ldo, n, w.rows,
                             w.k, ln.stream),
               "q8 GEMM");
    }

    // Both layer kinds run the tensor-core attention through maps whose token
    // extent is this wave's N (captured into its graph).
    void attention_maps(const Lane &ln, int N, AttnTcMaps (&tc_maps)[2]) {
        if (!exact && (!attention_tc_maps(&tc_maps[0], ln.qh, ln.kh, ln.vh, N, 256) ||
                       !attention_tc_maps(&tc_maps[1], ln.qh, ln.kh, ln.vh, N, 512)))
            ck(cudaErrorInvalidValue, "attention maps");
    }

    // Layer l of the wave (gemma2_fast.c:957-992): its first GEMM reads the Q8
    // operand of attn_norm(x) already in xq/xs; its last kernel leaves the next
    // layer's operand (or the output head's) there.  Returns kernels launched.
    template <class Mark>
    int enqueue_layer(int l, int N, Lane &ln, const AttnTcMaps (&tc_maps)[2], Mark &&mark) {
        int launches = 0;
        const Layer &L = layers[l];
        const int rb = L.d == 512 ? 1 : 0;
        cudaStream_t s = ln.stream;
        gemm(ln, L.qkv, ln.qkv, L.qkv.rows, N), ++launches;
        mark("gemm_qkv");
        if (exact) {
            ck(launch_qkv_post(ln.qf, ln.kf, ln.vf, ln.qkv, L.q_norm, L.k_norm, rope_cos[rb], rope_sin[rb], ln.pos, N,
                               L.d, s, true, tier),
               "qkv_post"),
                ++launches;
            mark("qkv_post");
            ck(launch_attention_exact(ln.attn, ln.qf, ln.kf, ln.vf, ln.bounds, N, L.d, L.d == 512 ? 0 : 512, s, tier),
               "attention"),
                ++launches;
        } else {
            ck(launch_qkv_post(ln.qh, ln.kh, ln.vh, ln.qkv, L.q_norm, L.k_norm, rope_cos[rb], rope_sin[rb], ln.pos, N,
                               L.d, s, false),
               "qkv_post"),
                ++launches;
            mark("qkv_post");
            // The O projection's Q8 operand is written by the attention itself.
            ck(launch_attention_tc(tc_maps[L.d == 512], nullptr, ln.bounds, N, L.d == 512 ? 0 : 512, s, ln.xq, ln.xs,
                                   cap, tier),
               "attention");
            ++launches;
        }
        mark(L.d == 512 ? "attention_global" : "attention_local");
        if (exact) {
            ck(launch_norm_quant(ln.xq, ln.xs, cap, nullptr, ln.attn, nullptr, N, 4 * L.d, s, tier), "quant"),
                ++launches;
            mark("quant_attn");
        }
        gemm(ln, L.o, ln.h, 512, N), ++launches;
        mark("gemm_o");
        ck(launch_post_add(ln.x, ln.h, L.post_attn_norm, nullptr, ln.xq, ln.xs, cap, L.ffn_norm, N, s, tier),
           "post_add"),
            ++launches;
        mark("post_add");
        // ffn_gate and ffn_up in one GEMM whose epilogue applies gelu(gate) * up
        // and quantizes (ROW_GELU_QUANT fused); the result is the down operand.
        if (vnni()) {  // gate and up as the reference's two GEMMs, then ROW_GELU_QUANT
            ck(launch_q8gemm_vnni(L.gu.codes, L.gu.scales, ln.xq, ln.xs, int(cap), ln.qkv, ln.attn, 2048, N, L.gu.rows,
                                  L.gu.k, ln.offsets, ln.seq_count, s),
               "GeGLU GEMM");
            ck(launch_gate_quant(ln.gq, ln.gs, cap, ln.qkv, ln.attn, N, 2048, 2048, 0, s, tier), "GELU quant");
            launches += 2;
        } else {
            ck(launch_q8gemm_geglu(L.gu.tmap, ln.tm_xq[0], L.gu.tscale, ln.tm_xs[0], exact, ln.gq, ln.gs, cap, N,
                                   L.gu.rows, L.gu.k, s, tier),
               "GeGLU GEMM"),
                ++launches;
        }
        mark("gemm_geglu");
        if (vnni())
            ck(launch_q8gemm_vnni(L.down.codes, L.down.scales, ln.gq, ln.gs, int(cap), ln.h, nullptr, 512, N,
                                  L.down.rows, L.down.k, ln.offsets, ln.seq_count, s),
               "q8 GEMM");
        else
            ck(launch_q8gemm(L.down.tmap, ln.tm_gq, L.down.tscale, ln.tm_gs, exact, ln.h, 512, N, L.down.rows,
                             L.down.k, s),
               "q8 GEMM");
        ++launches;
        mark("gemm_down");
        ck(launch_post_add(ln.x, ln.h, L.post_ffw_norm, nullptr, ln.xq, ln.xs, cap, nullptr, N, s, tier), "post_add"),
            ++launches;
        mark("post_add");
        gemm(ln, L.inp_gate, ln.h, 512, N), ++launches;
        mark("gemm_inp_gate");
        ck(launch_gate_quant(ln.xq, ln.xs, cap, ln.h, ln.ple, N, 512, 24 * 512, l * 512, s, tier), "ple gate"),
            ++launches;
        mark("ple_gate_quant");
        gemm(ln, L.proj, ln.h, 512, N), ++launches;
        mark("gemm_proj");
        const float *next = l + 1 < 24 ? layers[l + 1].attn_norm : output_norm;
        ck(launch_post_add(ln.x, ln.h, L.post_norm, L.out_scale, ln.xq, ln.xs, cap, next, N, s, tier), "post_add"),
            ++launches;
        mark("post_add");
        return launches;
    }

    // The whole wave as a launch sequence on a lane (captured into a graph, or
    // run eagerly under the profiler).  Returns the number of kernels launched.
    // rows: a soft-token wave, whose x was uploaded with the inputs.
    int enqueue(unsigned n, Lane &ln, Profiler *prof, bool rows = false) {
        int launches = 0;
        auto mark = [&](const char *name) {
            if (prof) prof->mark(name);
        };
        const int N = int(n);
        cudaStream_t s = ln.stream;
        AttnTcMaps tc_maps[2]{};
        attention_maps(ln, N, tc_maps);
        mark("start");
        if (rows)
            ck(launch_input_rows(ln.x, ln.x_hi, ln.x_lo, ln.xin, N, s), "input rows"), ++launches;
        else
            ck(launch_embed(ln.x, ln.x_hi, ln.x_lo, token_embd, ln.ids, N, s), "embed"), ++launches;
        mark("embed");
        if (exact)
            ck(launch_ple_exact(ln.ple, ln.x, ple_w, ple_norm, N, s, tier), "PLE"), launches += 2;
        else
            ck(launch_ple(ln.tm_hi, ln.tm_lo, tm_ple, ln.ple, ple_norm, N, s), "PLE"), ++launches;
        mark("ple_proj");
        ck(launch_norm_quant(ln.xq, ln.xs, cap, nullptr, ln.x, layers[0].attn_norm, N, 512, s, tier), "norm"),
            ++launches;
        mark("norm_quant");
        for (int l = 0; l < 24; ++l) launches += enqueue_layer(l, N, ln, tc_maps, mark);
        gemm(ln, output, ln.y, 768, N), ++launches;
        mark("gemm_output");
        // The grid covers every sequence a wave of n tokens can hold; the
        // wave's own count is read on the device.
        ck(launch_pool_l2(ln.pooled, ln.y, ln.offsets, int(n), 768, s, ln.seq_count), "pool"), launches += 2;
        mark("pool_l2");
        return launches;
    }

    cudaGraphExec_t graph_for(Lane &ln, unsigned n, bool rows = false) {
        const uint64_t key = n | uint64_t(rows) << 32;
        auto it = ln.graphs.find(key);
        if (it != ln.graphs.end()) return it->second;
        // Keys are (bucketed token count, ids or rows): at most 2 * cap / BUCKET
        // = 256 for the widest context, so this flush only guards the bound.
        if (ln.graphs.size() >= 256) {
            ck(cudaStreamSynchronize(ln.stream), "graph cache flush");
            for (auto &kv : ln.graphs) cudaGraphExecDestroy(kv.second);
            ln.graphs.clear();
            ln.staged_graph = nullptr;
            staged = false;  // stage() again before launch()
        }
        cudaGraph_t graph = nullptr;
        ck(cudaStreamBeginCapture(ln.stream, cudaStreamCaptureModeThreadLocal), "begin capture");
        int launches = 0;
        try {
            launches = enqueue(n, ln, nullptr, rows);
        } catch (...) {
            cudaStreamEndCapture(ln.stream, &graph);
            if (graph) cudaGraphDestroy(graph);
            throw;
        }
        ck(cudaStreamEndCapture(ln.stream, &graph), "end capture");
        cudaGraphExec_t exec = nullptr;
        const cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        ck(e, "graph instantiate");
        kernels_per_wave = launches;
        ln.graphs[key] = exec;
        return exec;
    }

    // gemma2_kfd.cpp:271-296: validation, bounds and positions into a lane's
    // staging buffer, padded to the bucket, and the upload on its stream;
    // returns the padded token count.  A soft-token wave (in_rows set, in_ids
    // NULL) uploads its rows, padded with zero rows to the bucket, into xin
    // (allocated on first use).
    unsigned fill(Lane &ln, const int32_t *in_ids, const size_t *in_off, size_t batch,
                  const float *in_rows = nullptr) {
        if (in_rows) validate_rows(in_rows, in_off, batch, cap);
        else validate_wave(in_ids, in_off, batch, cap);
        const unsigned n = unsigned(in_off[batch]);
        uint32_t *hid = ln.in, *hb = ln.in + cap, *hp = ln.in + 3 * cap, *ho = ln.in + 4 * cap;  // device layout
        if (in_ids && !in_rows) std::memcpy(hid, in_ids, n * sizeof(int32_t));
        else std::memset(hid, 0, n * sizeof(int32_t));
        for (size_t s = 0; s < batch; ++s) {
            ho[s] = uint32_t(in_off[s]);
            for (size_t t = in_off[s]; t < in_off[s + 1]; ++t) {
                hb[2 * t] = uint32_t(in_off[s]), hb[2 * t + 1] = uint32_t(in_off[s + 1]);
                hp[t] = uint32_t(t - in_off[s]);
            }
        }
        ho[batch] = n;
        // Padding to the bucket: one sequence [n, n_pad) of token 0, never pooled.
        const unsigned n_pad = (n + BUCKET - 1) / BUCKET * BUCKET;
        for (unsigned t = n; t < n_pad; ++t) hid[t] = 0, hb[2 * t] = n, hb[2 * t + 1] = n_pad, hp[t] = t - n;
        ln.in[5 * cap + 1] = uint32_t(batch);
        ck(cudaSetDevice(device), "cudaSetDevice");
        if (in_rows) {
            if (!ln.rows) ck(cudaMallocHost(&ln.rows, sizeof(float) * cap * 512), "cudaMallocHost");
            if (!ln.xin) ln.xin = dalloc<float>(size_t(cap) * 512);
            std::memcpy(ln.rows, in_rows, size_t(n) * 512 * sizeof(float));
            std::memset(ln.rows + size_t(n) * 512, 0, size_t(n_pad - n) * 512 * sizeof(float));
            ck(cudaMemcpyAsync(ln.xin, ln.rows, size_t(n_pad) * 512 * sizeof(float), cudaMemcpyHostToDevice,
                               ln.stream),
               "input rows upload");
        }
        ck(cudaMemcpyAsync(ln.ids, ln.in, (5 * cap + 2) * 4, cudaMemcpyHostToDevice, ln.stream), "wave upload");
        return n_pad;
    }

    // Capture the token-id wave graphs of every 64-token bucket up to
    // max_tokens (clamped to the context's cap) on every lane; returns how
    // many graphs exist afterwards.
    int prepare(unsigned max_tokens) {
        refuse_if_poisoned();
        refuse_if_submitted();
        if (max_tokens > cap) max_tokens = cap;
        ck(cudaSetDevice(device), "cudaSetDevice");
        for (Lane &ln : lanes)
            for (unsigned n = BUCKET; n <= max_tokens; n += BUCKET) graph_for(ln, n, false);
        int total = 0;
        for (const Lane &ln : lanes) total += int(ln.graphs.size());
        return total;
    }

    void refuse_if_poisoned() const {
        if (poisoned) throw std::runtime_error("KFD context failed; restart process before reuse");
    }
    void refuse_if_submitted() const {
        for (const Lane &ln : lanes)
            if (ln.busy) throw std::runtime_error("a submitted wave is not collected yet");
    }

    // Split form for device-resident timing: stage the wave into every lane
    // once, launch the staged graphs any number of times, finish.  Not to be
    // interleaved with submit/collect.
    void stage(const int32_t *in_ids, const size_t *in_off, size_t batch, const float *in_rows = nullptr) {
        refuse_if_poisoned();
        refuse_if_submitted();
        // Nothing stays staged if a fill or a capture below fails.
        staged = false;
        for (Lane &ln : lanes) ln.staged_graph = nullptr;
        unsigned n_pad = 0;
        for (Lane &ln : lanes) {
            n_pad = fill(ln, in_ids, in_off, batch, in_rows);
            ln.staged_graph = graph_for(ln, n_pad, in_rows != nullptr);
        }
        staged_n = n_pad, staged_batch = batch, staged_rows = in_rows != nullptr;
        staged = true;
    }

    // Replays alternate over the lanes (replay r on lane r % LANES), so
    // consecutive waves overlap on the GPU as two submitted waves do.  The
    // other lanes start after the work already queued on the first lane's
    // stream, and the first lane's stream waits for them at the end: events
    // recorded on that stream (eg2_b200_stream) around a launch bracket all
    // of its replays.  One replay runs on the first lane alone.
    void launch(int repeats) {
        refuse_if_poisoned();
        if (!staged) throw std::runtime_error("no wave staged");
        const int used = repeats < LANES ? repeats : LANES;
        if (used > 1) {
            ck(cudaEventRecord(lanes[0].fork, lanes[0].stream), "event record");
            for (int i = 1; i < used; ++i) ck(cudaStreamWaitEvent(lanes[i].stream, lanes[0].fork, 0), "stream wait");
        }
        for (int r = 0; r < repeats; ++r) {
            Lane &ln = lanes[r % LANES];
            ck(cudaGraphLaunch(ln.staged_graph, ln.stream), "graph launch");
        }
        for (int i = 1; i < used; ++i) {
            ck(cudaEventRecord(lanes[i].join, lanes[i].stream), "event record");
            ck(cudaStreamWaitEvent(lanes[0].stream, lanes[i].join, 0), "stream wait");
        }
    }

    // Enqueue a lane's readback (embeddings, error word) and completion event.
    void enqueue_readback(Lane &ln, size_t batch) {
        if (batch)
            ck(cudaMemcpyAsync(ln.out, ln.pooled, batch * 768 * 4, cudaMemcpyDeviceToHost, ln.stream), "readback");
        ck(read_device_error_async(ln.err, ln.stream), "error readback");
        ck(cudaEventRecord(ln.done, ln.stream), "event record");
    }

    // Wait for a lane with the reference's deadline.  Any failure poisons the
    // context for good (gemma2_kfd.cpp:190-214): a later wait that succeeds,
    // e.g. the other pipeline slot's, never clears it.
    void wait_lane(Lane &ln) {
        try {
            // Poll without sleeping for the length of a few waves, then back off.
            const auto t0 = std::chrono::steady_clock::now();
            for (;;) {
                const cudaError_t q = cudaEventQuery(ln.done);
                if (q == cudaSuccess) break;
                if (q != cudaErrorNotReady) ck(q, "GPU wave");
                const double waited = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
                if (waited > TIMEOUT_S) throw std::runtime_error("GPU wave timed out");
                if (waited > 0.02) std::this_thread::sleep_for(std::chrono::microseconds(50));
            }
            const int derr = *ln.err;
            if (derr)
                throw std::runtime_error("device wait timed out inside a kernel (error " + std::to_string(derr) + ")");
        } catch (...) {
            poisoned = true;
            throw;
        }
    }

    // gemma2_kfd.cpp:337-343: finite, non-zero; the embedding is already
    // L2-normalised on the device.
    void deliver(const Lane &ln, size_t batch, float *out) {
        for (size_t s = 0; s < batch; ++s) {
            double ss = 0;
            for (int z = 0; z < 768; ++z) {
                const float f = ln.out[s * 768 + z];
                if (!std::isfinite(f)) throw std::runtime_error("nonfinite GPU output");
                ss += double(f) * f;
            }
            if (ss <= 0) throw std::runtime_error("zero GPU embedding");
        }
        std::memcpy(out, ln.out, batch * 768 * sizeof(float));
    }

    void finish(float *out) {
        refuse_if_poisoned();
        if (!staged) throw std::runtime_error("no wave staged");
        enqueue_readback(lanes[0], staged_batch);
        wait_lane(lanes[0]);
        deliver(lanes[0], staged_batch, out);
    }

    // Pipelined form: submit enqueues upload, graph and readback on the next
    // slot's lane and returns the slot index; collect waits for that slot and
    // delivers.  A slot must be collected before it is submitted to again.
    int submit(const int32_t *in_ids, const size_t *in_off, size_t batch, const float *in_rows = nullptr) {
        refuse_if_poisoned();
        // The next slot in turn, or the other one if a synchronous call holds it.
        int id = next_slot;
        for (int i = 0; i < LANES && lanes[id].busy; ++i) id = (next_slot + i + 1) % LANES;
        Lane &ln = lanes[id];
        if (ln.busy) throw std::runtime_error("pipeline slot busy: collect its wave first");
        staged = false;  // the staged wave's device inputs on this lane are overwritten
        const unsigned n_pad = fill(ln, in_ids, in_off, batch, in_rows);
        ck(cudaGraphLaunch(graph_for(ln, n_pad, in_rows != nullptr), ln.stream), "graph launch");
        enqueue_readback(ln, batch);
        ln.batch = batch, ln.busy = true;
        next_slot = (id + 1) % LANES;
        return id;
    }

    void collect(int id, float *out) {
        if (id < 0 || id >= LANES || !lanes[id].busy || lanes[id].by_call)
            throw std::runtime_error("no wave submitted to this slot");
        Lane &ln = lanes[id];
        ln.busy = false;
        refuse_if_poisoned();
        wait_lane(ln);
        deliver(ln, ln.batch, out);
    }

    // The synchronous call (ei_gemma2_kfd_batch), safe to make from several
    // host threads at once: it holds the context's mutex only to enqueue the
    // wave on a free lane and to deliver it, not while the GPU runs it, so two
    // callers' waves overlap on the GPU.  A third caller waits for a lane
    // (up to the wave deadline).  Takes the mutex itself.
    void batch(const int32_t *in_ids, const size_t *in_off, size_t n_seq, float *out, const float *in_rows = nullptr) {
        std::unique_lock<std::mutex> lk(mutex);
        if (!out) throw std::runtime_error(count_message(cap));
        refuse_if_poisoned();
        Lane *ln = nullptr;
        auto free_lane = [&] {
            for (Lane &l : lanes)
                if (!l.busy) return ln = &l, true;
            return poisoned.load();
        };
        if (!lane_freed.wait_for(lk, std::chrono::duration<double>(TIMEOUT_S), free_lane))
            throw std::runtime_error("GPU wave timed out");
        refuse_if_poisoned();
        staged = false;  // the staged wave's device inputs on this lane are overwritten
        const unsigned n_pad = fill(*ln, in_ids, in_off, n_seq, in_rows);
        ck(cudaGraphLaunch(graph_for(*ln, n_pad, in_rows != nullptr), ln->stream), "graph launch");
        enqueue_readback(*ln, n_seq);
        ln->busy = ln->by_call = true;
        lk.unlock();
        std::exception_ptr failure;
        try {
            wait_lane(*ln);
        } catch (...) {
            failure = std::current_exception();
        }
        lk.lock();
        try {
            if (failure) std::rethrow_exception(failure);
            deliver(*ln, n_seq, out);
        } catch (...) {
            ln->busy = ln->by_call = false;
            lane_freed.notify_all();
            throw;
        }
        ln->busy = ln->by_call = false;
        lane_freed.notify_all();
    }

    // Layers [l0, l1) of the fast path (or of parity mode) from a caller-given
    // residual stream x_in [n][512] and per-layer embeddings ple_in
    // [n][24][512] (NULL: projected on the device from x_in, which is then the
    // wave's embedding rows), eager launches on the first lane's stream; x_out
    // gets the residual stream after layer l1 - 1.  For teacher-forced
    // per-layer checks against the reference CPU graph.
    void forward_layers(const float *x_in, const float *ple_in, const size_t *in_off, size_t batch, int l0, int l1,
                        float *x_out) {
        refuse_if_poisoned();
        refuse_if_submitted();
        if (l0 < 0 || l1 > 24 || l0 > l1 || !x_out) throw std::runtime_error("invalid layer range");
        staged = false;  // the staged wave's device inputs are overwritten below
        Lane &ln = lanes[0];
        const unsigned n_pad = fill(ln, nullptr, in_off, batch, x_in);
        const int N = int(n_pad);
        const size_t n = in_off[batch];
        cudaStream_t s = ln.stream;
        ck(launch_input_rows(ln.x, ln.x_hi, ln.x_lo, ln.xin, N, s), "input rows");
        if (ple_in) {
            ck(cudaMemcpyAsync(ln.ple, ple_in, n * 24 * 512 * sizeof(float), cudaMemcpyHostToDevice, s),
               "PLE upload");
            ck(cudaStreamSynchronize(s), "PLE upload");  // ple_in is pageable caller memory
        } else if (exact) {
            ck(launch_ple_exact(ln.ple, ln.x, ple_w, ple_norm, N, s, tier), "PLE");
        } else {
            ck(launch_ple(ln.tm_hi, ln.tm_lo, tm_ple, ln.ple, ple_norm, N, s), "PLE");
        }
        AttnTcMaps tc_maps[2]{};
        attention_maps(ln, N, tc_maps);
        if (l0 < 24)
            ck(launch_norm_quant(ln.xq, ln.xs, cap, nullptr, ln.x, layers[l0].attn_norm, N, 512, s, tier), "norm");
        auto none = [](const char *) {};
        for (int l = l0; l < l1; ++l) enqueue_layer(l, N, ln, tc_maps, none);
        enqueue_readback(ln, 0);
        wait_lane(ln);
        ck(cudaMemcpy(x_out, ln.x, n * 512 * sizeof(float), cudaMemcpyDeviceToHost), "residual readback");
    }

    int profile(char names[][32], double *ms, int max) {
        refuse_if_poisoned();
        if (!staged) throw std::runtime_error("no wave staged");
        std::map<std::string, double> acc;
        std::vector<std::string> order;
        {
            Profiler prof{lanes[0].stream};
            enqueue(staged_n, lanes[0], &prof, staged_rows);
            enqueue_readback(lanes[0], 0);
            wait_lane(lanes[0]);
            for (size_t i = 1; i < prof.events.size(); ++i) {
                float t = 0;
                ck(cudaEventElapsedTime(&t, prof.events[i - 1], prof.events[i]), "elapsed");
                if (!acc.count(prof.names[i])) order.push_back(prof.names[i]);
                acc[prof.names[i]] += t;
            }
        }
        int k = 0;
        for (auto &nm : order) {
            if (k >= max) break;
            std::snprintf(names[k], 32, "%s", nm.c_str());
            ms[k++] = acc[nm];
        }
        return k;
    }
};

template <class F>
bool guarded(char *err, size_t len, F &&f) {
    try {
        f();
        return true;
    } catch (const std::exception &e) {
        if (err && len) std::snprintf(err, len, "KFD: %s", e.what());
        return false;
    }
}
Backend *as_backend(void *ctx) {
    if (!ctx) throw std::runtime_error("empty context");
    return static_cast<Backend *>(ctx);
}
}  // namespace

extern "C" void *eg2_b200_create(const ei_gguf *g, int device, unsigned flags, char *err, size_t len) {
    Backend *b = nullptr;
    guarded(err, len, [&] { b = new Backend(g, device, flags); });
    return b;
}
extern "C" void *ei_gemma2_kfd_create_on(const ei_gguf *g, int device, char *err, size_t len) {
    return eg2_b200_create(g, device, 0u, err, len);
}
extern "C" void *ei_gemma2_kfd_create(const ei_gguf *g, char *err, size_t len) {
    const char *env = std::getenv("EG2_B200_DEVICE");
    return ei_gemma2_kfd_create_on(g, env ? std::atoi(env) : 0, err, len);
}
extern "C" void ei_gemma2_kfd_free(void *ctx) { delete static_cast<Backend *>(ctx); }
extern "C" bool ei_gemma2_kfd_batch(void *ctx, const int32_t *ids, const size_t *offsets, size_t batch, float *out,
                                    char *err, size_t len) {
    return guarded(err, len, [&] {
        as_backend(ctx)->batch(ids, offsets, batch, out);
    });
}
extern "C" bool eg2_b200_validate(const int32_t *ids, const size_t *offsets, size_t batch, char *err, size_t len) {
    return guarded(err, len, [&] { validate_wave(ids, offsets, batch); });
}
extern "C" bool eg2_b200_stage(void *ctx, const int32_t *ids, const size_t *offsets, size_t batch, char *err,
                               size_t len) {
    return guarded(err, len, [&] {
        Backend *b = as_backend(ctx);
        std::lock_guard<std::mutex> guard(b->mutex);
        b->stage(ids, offsets, batch);
    });
}
extern "C" bool eg2_b200_launch(void *ctx, int repeats, char *err, size_t len) {
    return guarded(err, len, [&] {
        Backend *b = as_backend(ctx);
        std::lock_guard<std::mutex> guard(b->mutex);
        ck(cudaSetDevice(b->device), "cudaSetDevice");
        b->launch(repeats);
    });
}
extern "C" bool eg2_b200_finish(void *ctx, float *out, char *err, size_t len) {
    return guarded(err, len, [&] {
        Backend *b = as_backend(ctx);
        std::lock_guard<std::mutex> guard(b->mutex);
        if (!out) throw std::runtime_error("null output");
        ck(cudaSetDevice(b->device), "cudaSetDevice");
        b->finish(out);
    });
}
extern "C" int eg2_b200_submit(void *ctx, const int32_t *ids, const size_t *offsets, size_t batch, char *err,
                               size_t len) {
    int slot = -1;
    guarded(err, len, [&] {
        Backend *b = as_backend(ctx);
        std::lock_guard<std::mutex> guard(b->mutex);
        slot = b->submit(ids, offsets, batch);
    });
    return slot;
}
extern "C" bool eg2_b200_collect(void *ctx, int slot, float *out, char *err, size_t len) {
    return guarded(err, len, [&] {
        Backend *b = as_backend(ctx);
        std::lock_guard<std::mutex> guard(b->mutex);
        if (!out) throw std::runtime_error("null output");
        ck(cudaSetDevice(b->device), "cudaSetDevice");
        b->collect(slot, out);
    });
}
extern "C" bool eg2_b200_validate_rows(const float *rows, const size_t *offsets, size_t batch, char *err,
                                       size_t len) {
    return guarded(err, len, [&] { validate_rows(rows, offsets, batch); });
}
extern "C" bool eg2_b200_batch_rows(void *ctx, const float *rows, const size_t *offsets, size_t batch, float *out,
                                    char *err, size_t len) {
    return guarded(err, len, [&] {
        Backend *b = as_backend(ctx);
        if (!rows) throw std::runtime_error(count_message(b->cap));
        b->batch(nullptr, offsets, batch, out, rows);
    });
}
extern "C" bool eg2_b200_stage_rows(void *ctx, const float *rows, const size_t *offsets, size_t batch, char *err,
                                    size_t len) {
    return guarded(err, len, [&] {
        Backend *b = as_backend(ctx);
        std::lock_guard<std::mutex> guard(b->mutex);
        if (!rows) throw std::runtime_error(count_message(b->cap));
        b->stage(nullptr, offsets, batch, rows);
    });
}
extern "C" int eg2_b200_submit_rows(void *ctx, const float *rows, const size_t *offsets, size_t batch, char *err,
                                    size_t len) {
    int slot = -1;
    guarded(err, len, [&] {
        Backend *b = as_backend(ctx);
        std::lock_guard<std::mutex> guard(b->mutex);
        if (!rows) throw std::runtime_error(count_message(b->cap));
        slot = b->submit(nullptr, offsets, batch, rows);
    });
    return slot;
}
extern "C" bool eg2_b200_forward_layers(void *ctx, const float *x_in, const float *ple_in, const size_t *offsets,
                                        size_t batch, int first_layer, int last_layer, float *x_out, char *err,
                                        size_t len) {
    return guarded(err, len, [&] {
        Backend *b = as_backend(ctx);
        std::lock_guard<std::mutex> guard(b->mutex);
        if (!x_in) throw std::runtime_error(count_message(b->cap));
        b->forward_layers(x_in, ple_in, offsets, batch, first_layer, last_layer, x_out);
    });
}
// Matryoshka truncation as the server applies it (kernels.c:398-407,
// server.c:1133): keep the first dims of a 768-wide L2-normalised embedding
// and, when shorter, renormalise with the sum of squares in the order of the
// server's SSE2 build (kernels.c:82-93: two 4-lane accumulators over 8-element
// chunks, then (v0 + v2) + (v1 + v3), kernels.c:35-39) and x *= 1 / sqrtf(ss)
// (kernels.c:393-396).  Plain host arithmetic: products and sums rounded one
// by one, no contraction (baseline x86-64 has no FMA).
extern "C" bool eg2_b200_normalize_prefix(float *x, int dims) {
    if (!x || (dims != 128 && dims != 256 && dims != 512 && dims != 768)) return false;
    if (dims == 768) return true;
    float s0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, s1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int i = 0;
    for (; i + 7 < dims; i += 8)
        for (int j = 0; j < 4; ++j) {
            const float a = x[i + j] * x[i + j], b = x[i + 4 + j] * x[i + 4 + j];
            s0[j] = s0[j] + a;
            s1[j] = s1[j] + b;
        }
    float v[4];
    for (int j = 0; j < 4; ++j) v[j] = s0[j] + s1[j];
    float ss = (v[0] + v[2]) + (v[1] + v[3]);
    for (; i < dims; ++i) {
        const float a = x[i] * x[i];
        ss = ss + a;
    }
    if (ss != 0.0f) {
        const float sc = 1.0f / std::sqrt(ss);
        for (int z = 0; z < dims; ++z) x[z] *= sc;
    }
    return true;
}
extern "C" void *eg2_b200_stream(void *ctx) { return ctx ? static_cast<Backend *>(ctx)->stream : nullptr; }
extern "C" int eg2_b200_prepare(void *ctx, unsigned max_tokens, char *err, size_t len) {
    int total = -1;
    guarded(err, len, [&] {
        Backend *b = as_backend(ctx);
        std::lock_guard<std::mutex> guard(b->mutex);
        total = b->prepare(max_tokens);
    });
    return total;
}
extern "C" int eg2_b200_kernels_per_wave(void *ctx) { return ctx ? static_cast<Backend *>(ctx)->kernels_per_wave : 0; }
extern "C" int eg2_b200_device(void *ctx) { return ctx ? static_cast<Backend *>(ctx)->device : -1; }
extern "C" int eg2_b200_profile(void *ctx, char names[][32], double *ms, int max) {
    int k = -1;
    guarded(nullptr, 0, [&] {
        Backend *b = as_backend(ctx);
        std::lock_guard<std::mutex> guard(b->mutex);
        ck(cudaSetDevice(b->device), "cudaSetDevice");
        k = b->profile(names, ms, max);
    });
    return k;
}

// ---------------------------------------------------------------- the reference's CUDA executor ABI
// include/gemma2_cuda.h: the entry points of vendor/embeddinggemma.c/src/
// gemma2_cuda.h:13-33 on this executor, so the reference's engine and server
// built for their CUDA backend (several devices, pipeline slots) run on it.
// A handle is a context (owner) or a pipeline-slot clone of one; clones share
// the owner's Backend, whose two lanes already run two calls' waves at once.
namespace {
struct CudaHandle {
    Backend *b;
    bool owner;
};
// Errors as the reference's CUDA executor reports them: no "KFD: " prefix.
template <class F>
bool guarded_cuda(char *err, size_t len, F &&f) {
    try {
        f();
        return true;
    } catch (const std::exception &e) {
        if (err && len) std::snprintf(err, len, "%s", e.what());
        return false;
    }
}
CudaHandle *as_cuda(void *ctx) {
    if (!ctx) throw std::runtime_error("empty context");
    return static_cast<CudaHandle *>(ctx);
}
constexpr size_t CUDA_WAVE = 8192;  // gemma2_cuda.cu:717
}  // namespace

extern "C" int ei_gemma2_cuda_device_count(void) {
    int count = 0;
    return cudaGetDeviceCount(&count) == cudaSuccess ? count : 0;
}
extern "C" void *ei_gemma2_cuda_create_on(const ei_gguf *g, int device, char *err, size_t len) {
    CudaHandle *h = nullptr;
    guarded_cuda(err, len, [&] {
        const int count = ei_gemma2_cuda_device_count();
        if (count == 0) throw std::runtime_error("no CUDA device");
        if (device < 0 || device >= count)
            throw std::runtime_error("CUDA device " + std::to_string(device) + " does not exist (" +
                                     std::to_string(count) + " visible)");
        Backend *b = new Backend(g, device, EG2_B200_WAVE_8192);
        h = new CudaHandle{b, true};
    });
    return h;
}
extern "C" void *ei_gemma2_cuda_create(const ei_gguf *g, char *err, size_t len) {
    const char *env = std::getenv("EI_CUDA_DEVICE");
    return ei_gemma2_cuda_create_on(g, env ? std::atoi(env) : 0, err, len);
}
extern "C" int ei_gemma2_cuda_device(void *ctx) { return ctx ? static_cast<CudaHandle *>(ctx)->b->device : -1; }
extern "C" void ei_gemma2_cuda_free(void *ctx) {
    CudaHandle *h = static_cast<CudaHandle *>(ctx);
    if (!h) return;
    if (h->owner) delete h->b;
    delete h;
}
extern "C" void *ei_gemma2_cuda_clone(void *ctx, bool high_priority, char *err, size_t len) {
    (void)high_priority;
    CudaHandle *h = nullptr;
    guarded_cuda(err, len, [&] { h = new CudaHandle{as_cuda(ctx)->b, false}; });
    return h;
}
extern "C" bool ei_gemma2_cuda_batch(void *ctx, const int32_t *ids, const size_t *offsets, size_t batch, float *out,
                                     char *err, size_t len) {
    return guarded_cuda(err, len, [&] {
        Backend *b = as_cuda(ctx)->b;
        if (!offsets || !out) throw std::runtime_error("EmbeddingGemma 2 accepts 1..8192 tokens per wave");
        // Waves above 8192 tokens are split at sequence boundaries (gemma2_cuda.cu:1455-1467).
        std::vector<size_t> local;
        for (size_t first = 0; first < batch;) {
            size_t last = first + 1;
            while (last < batch && offsets[last + 1] - offsets[first] <= CUDA_WAVE) last++;
            const size_t n = offsets[last] - offsets[first];
            if (!n || n > CUDA_WAVE) throw std::runtime_error("EmbeddingGemma 2 accepts 1..8192 tokens per wave");
            local.assign(last - first + 1, 0);
            for (size_t s = first; s <= last; ++s) local[s - first] = offsets[s] - offsets[first];
            b->batch(ids ? ids + offsets[first] : nullptr, local.data(), last - first, out + first * 768);
            first = last;
        }
    });
}
extern "C" bool ei_gemma2_cuda_embed_inputs(void *ctx, const float *inputs, size_t n, float out[768], char *err,
                                            size_t len) {
    return guarded_cuda(err, len, [&] {
        if (!inputs || !n || n > CUDA_WAVE)
            throw std::runtime_error("EmbeddingGemma 2 accepts 1..8192 tokens per wave");
        const size_t offsets[2] = {0, n};
        as_cuda(ctx)->b->batch(nullptr, offsets, 1, out, inputs);
    });
}
extern "C" bool ei_gemma2_cuda_vision(void *ctx, const ei_gguf *projector, const uint8_t *rgb, int width,
                                      int height, float **out, size_t *tokens, char *err, size_t len) {
    (void)ctx, (void)projector, (void)rgb, (void)width, (void)height, (void)out, (void)tokens;
    if (err && len)
        std::snprintf(err, len, "the image tower is not part of the B200 executor; embed its soft tokens with "
                                "ei_gemma2_cuda_embed_inputs");
    return false;
}
extern "C" bool ei_gemma2_cuda_audio(void *ctx, const ei_gguf *projector, const float *mel, int frames, float **out,
                                     size_t *tokens, char *err, size_t len) {
    (void)ctx, (void)projector, (void)mel, (void)frames, (void)out, (void)tokens;
    if (err && len)
        std::snprintf(err, len, "the audio tower is not part of the B200 executor; embed its soft tokens with "
                                "ei_gemma2_cuda_embed_inputs");
    return false;
}
