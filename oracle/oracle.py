"""TEST INFRASTRUCTURE -- ctypes access to the two CPU checkers.

* `RefGraph`: the reference's OWN CPU graph compiled from its sources
  (oracle/_ref/libeg2ref.so, recipe in oracle/Makefile), driven through
  vendor/embeddinggemma.c/src/gemma2_fast.c:919 `ei_gemma2_embed_batch_fast_ctx`.
* `Port`: the plain-C restatement oracle/eg2_oracle.c (scalar tier), with
  per-operator entry points for the GPU operator tests.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline arm import
this module; the product never does.
"""
from __future__ import annotations

import ctypes as C
import os
import struct
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_SO = os.path.join(HERE, "_ref", "libeg2ref.so")
CUDA_REF_SO = os.path.join(HERE, "_ref", "libeg2cudaref.so")
ENGINE_LINK_SO = os.path.join(HERE, "_ref", "libeg2enginelink.so")
PORT_SO = os.path.join(HERE, "_build", "libeg2oracle.so")

GGML_F32, GGML_F16, GGML_Q8_0, GGML_BF16 = 0, 1, 8, 30


def ref_root() -> str:
    """The reference tree: $REF_ROOT, else a directory `reference` beside this
    repository's root (the oracle's Makefile uses the same default)."""
    return os.environ.get("REF_ROOT") or os.path.abspath(os.path.join(HERE, "..", "..", "reference"))


def build(ref: bool = True, cuda: bool = True) -> None:
    """Compile the restatement, and the reference (its CPU graph, with cuda
    its CUDA executor, and, once libeg2_b200.so exists, its engine and HTTP
    server linked with it) when its sources exist."""
    subprocess.run(["make", "-s", "-C", HERE, "port"], check=True)
    root = ref_root()
    if ref and os.path.isdir(os.path.join(root, "vendor")):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF_ROOT={root}"], check=True)
        if cuda:
            subprocess.run(["make", "-s", "-C", HERE, "cuda_ref", f"REF_ROOT={root}"], check=True)
        if os.path.exists(os.path.join(HERE, "..", "embeddinggemma2-amdkfd_b200", "libeg2_b200.so")):
            subprocess.run(["make", "-s", "-C", HERE, "engine_link", "server", f"REF_ROOT={root}"], check=True)


# ---------------------------------------------------------------------------
# GGUF v3 reader (numpy memmap), same format as vendor/embeddinggemma.c/src/gguf.c
# ---------------------------------------------------------------------------
class Gguf:
    def __init__(self, path: str):
        self.path = path
        self.map = np.memmap(path, dtype=np.uint8, mode="r")
        buf = self.map
        pos = 0

        def take(n):
            nonlocal pos
            b = bytes(buf[pos:pos + n])
            pos += n
            return b

        def u32():
            return struct.unpack("<I", take(4))[0]

        def u64():
            return struct.unpack("<Q", take(8))[0]

        def string():
            return take(u64()).decode()

        sizes = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}
        assert take(4) == b"GGUF" and u32() == 3
        n_t, n_kv = u64(), u64()
        self.kv = {}
        for _ in range(n_kv):
            key, typ = string(), u32()
            if typ == 8:
                self.kv[key] = string()
            elif typ == 9:
                at, n = u32(), u64()
                if at == 8:
                    self.kv[key] = [string() for _ in range(n)]
                else:
                    self.kv[key] = take(sizes[at] * n)
            else:
                raw = take(sizes[typ])
                self.kv[key] = int.from_bytes(raw, "little")
        align = int(self.kv.get("general.alignment", 32))
        infos = []
        for _ in range(n_t):
            name = string()
            nd = u32()
            ne = [u64() for _ in range(nd)] + [1] * (4 - nd)
            typ, off = u32(), u64()
            infos.append((name, ne, typ, off))
        data_off = (pos + align - 1) // align * align
        self.tensors = {}
        for name, ne, typ, off in infos:
            n = ne[0] * ne[1] * ne[2] * ne[3]
            nbytes = {GGML_F32: 4 * n, GGML_F16: 2 * n, GGML_BF16: 2 * n, GGML_Q8_0: n // 32 * 34}[typ]
            self.tensors[name] = (ne, typ, self.map[data_off + off: data_off + off + nbytes])

    def raw(self, name: str) -> np.ndarray:
        return self.tensors[name][2]

    def f32(self, name: str) -> np.ndarray:
        return self.raw(name).view(np.float32)

    def q8(self, name: str):
        """(int8 codes [rows][k], fp16 scale bits uint16 [rows][k/32])."""
        ne, typ, raw = self.tensors[name]
        assert typ == GGML_Q8_0
        blk = np.asarray(raw).reshape(-1, 34)
        d = np.ascontiguousarray(blk[:, :2]).view(np.uint16).reshape(ne[1], ne[0] // 32)
        q = np.ascontiguousarray(blk[:, 2:]).view(np.int8).reshape(ne[1], ne[0])
        return q, d

    def pointer_table(self):
        """Tensor pointers in the order oracle/eg2_oracle.h documents."""
        names = ["token_embd.weight", "per_layer_model_proj.weight", "per_layer_proj_norm.weight"]
        for l in range(24):
            names += [f"blk.{l}.{s}.weight" for s in (
                "attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "attn_q_norm",
                "attn_k_norm", "post_attention_norm", "ffn_norm", "ffn_up", "ffn_gate",
                "ffn_down", "post_ffw_norm", "inp_gate", "proj", "post_norm", "layer_output_scale")]
        names += ["output_norm.weight", "output.weight"]
        arr = (C.c_void_p * len(names))()
        for i, nm in enumerate(names):
            arr[i] = self.raw(nm).ctypes.data
        return arr


def _ptr(a: np.ndarray):
    return C.c_void_p(a.ctypes.data)


class RefGraph:
    """The reference's compiled CPU graph (gemma2_fast.c / gemma2.c)."""

    def __init__(self, model_path: str, threads: int = 0):
        if not os.path.exists(REF_SO):
            raise FileNotFoundError(f"{REF_SO} missing: run `make -C oracle ref` where the reference exists")
        self.lib = C.CDLL(REF_SO)
        L = self.lib
        L.eg2ref_open.restype = C.c_void_p
        L.eg2ref_open.argtypes = [C.c_char_p, C.c_int]
        L.eg2ref_close.argtypes = [C.c_void_p]
        L.eg2ref_threads.argtypes = [C.c_void_p]
        L.eg2ref_embed_fast.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p,
                                        C.c_char_p, C.c_size_t]
        L.eg2ref_embed_reference.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p,
                                             C.c_char_p, C.c_size_t]
        L.eg2ref_embed_fast_inputs.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p,
                                               C.c_char_p, C.c_size_t]
        L.eg2ref_normalize_prefix.argtypes = [C.c_void_p, C.c_int]
        L.eg2ref_quantize_row_q8_0.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
        L.eg2ref_fp32_to_fp16.argtypes = [C.c_float]
        L.eg2ref_fp32_to_fp16.restype = C.c_uint16
        L.eg2ref_gelu_mul_row.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
        self.handle = L.eg2ref_open(model_path.encode(), threads)
        self.threads = L.eg2ref_threads(self.handle)

    @property
    def tier(self) -> str:
        lvl = self.lib.eg2ref_x86_tier()
        name = {0: "scalar", 1: "avx2", 2: "avxvnni", 3: "vnni512"}.get(lvl, str(lvl))
        return name + ("+gemm512" if self.lib.eg2ref_x86_wide512() else "")

    def embed(self, ids: np.ndarray, offsets: np.ndarray) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        offsets = np.ascontiguousarray(offsets, dtype=np.uint64)
        batch = len(offsets) - 1
        out = np.zeros((batch, 768), np.float32)
        err = C.create_string_buffer(256)
        if not self.lib.eg2ref_embed_fast(self.handle, _ptr(ids), _ptr(offsets), batch, _ptr(out), err, 256):
            raise RuntimeError(err.value.decode())
        return out

    def embed_inputs(self, inputs: np.ndarray, offsets: np.ndarray) -> np.ndarray:
        """The reference's CPU graph from 512-wide input rows (ids NULL)."""
        inputs = np.ascontiguousarray(inputs, dtype=np.float32).reshape(-1, 512)
        offsets = np.ascontiguousarray(offsets, dtype=np.uint64)
        batch = len(offsets) - 1
        out = np.zeros((batch, 768), np.float32)
        err = C.create_string_buffer(256)
        if not self.lib.eg2ref_embed_fast_inputs(self.handle, _ptr(inputs), _ptr(offsets), batch, _ptr(out),
                                                 err, 256):
            raise RuntimeError(err.value.decode())
        return out

    def embed_reference_graph(self, ids: np.ndarray) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.zeros(768, np.float32)
        err = C.create_string_buffer(256)
        if not self.lib.eg2ref_embed_reference(self.handle, _ptr(ids), len(ids), _ptr(out), err, 256):
            raise RuntimeError(err.value.decode())
        return out

    def normalize_prefix(self, emb: np.ndarray, dims: int) -> np.ndarray:
        e = np.array(emb, dtype=np.float32, copy=True)
        if not self.lib.eg2ref_normalize_prefix(_ptr(e), dims):
            raise ValueError("unsupported dimensions")
        return e[:dims]

    def quantize_x86(self, x: np.ndarray):
        x = np.ascontiguousarray(x, dtype=np.float32)
        blk = np.zeros((x.size // 32, 34), np.uint8)
        self.lib.eg2ref_quantize_row_q8_0(_ptr(x), _ptr(blk), x.size)
        d = np.ascontiguousarray(blk[:, :2]).view(np.uint16).ravel()
        q = np.ascontiguousarray(blk[:, 2:]).view(np.int8).ravel()
        return q, d

    def gelu_mul(self, g: np.ndarray, u: np.ndarray | None) -> np.ndarray:
        g = np.array(g, dtype=np.float32, copy=True)
        u = np.ascontiguousarray(u, dtype=np.float32) if u is not None else None  # kept alive
        self.lib.eg2ref_gelu_mul_row(_ptr(g), _ptr(u) if u is not None else None, g.size)
        return g

    def close(self):
        if self.handle:
            self.lib.eg2ref_close(self.handle)
            self.handle = None


class CudaRef:
    """The reference's own CUDA executor for the same graph (gemma2_cuda.cu,
    compiled from its sources into oracle/_ref/libeg2cudaref.so): the GPU
    comparator, driven through its packed-wave call ei_gemma2_cuda_batch."""

    def __init__(self, model_path: str, device: int = 0):
        if not os.path.exists(CUDA_REF_SO):
            raise FileNotFoundError(f"{CUDA_REF_SO} missing: run `make -C oracle cuda_ref` where the reference exists")
        self.lib = C.CDLL(CUDA_REF_SO)
        L = self.lib
        L.eg2cref_open.restype = C.c_void_p
        L.eg2cref_open.argtypes = [C.c_char_p, C.c_int, C.c_char_p, C.c_size_t]
        L.eg2cref_close.argtypes = [C.c_void_p]
        L.eg2cref_batch.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_char_p,
                                    C.c_size_t]
        L.eg2cref_slot.restype = C.c_void_p
        L.eg2cref_slot.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t]
        L.eg2cref_slot_batch.argtypes = L.eg2cref_batch.argtypes
        L.eg2cref_slot_free.argtypes = [C.c_void_p]
        err = C.create_string_buffer(512)
        self.handle = L.eg2cref_open(model_path.encode(), device, err, 512)
        if not self.handle:
            raise RuntimeError(err.value.decode())
        self.slot = None

    def open_slot(self):
        """A second pipeline slot (ei_gemma2_cuda_clone): its own stream, so
        calls through it overlap calls through the first on the GPU."""
        err = C.create_string_buffer(512)
        self.slot = self.lib.eg2cref_slot(self.handle, err, 512)
        if not self.slot:
            raise RuntimeError(err.value.decode())

    def embed_slot(self, ids: np.ndarray, offsets: np.ndarray) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        offsets = np.ascontiguousarray(offsets, dtype=np.uint64)
        out = np.zeros((len(offsets) - 1, 768), np.float32)
        err = C.create_string_buffer(512)
        if not self.lib.eg2cref_slot_batch(self.slot, _ptr(ids), _ptr(offsets), len(offsets) - 1, _ptr(out), err,
                                           512):
            raise RuntimeError(err.value.decode())
        return out

    def embed(self, ids: np.ndarray, offsets: np.ndarray) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        offsets = np.ascontiguousarray(offsets, dtype=np.uint64)
        batch = len(offsets) - 1
        out = np.zeros((batch, 768), np.float32)
        err = C.create_string_buffer(512)
        if not self.lib.eg2cref_batch(self.handle, _ptr(ids), _ptr(offsets), batch, _ptr(out), err, 512):
            raise RuntimeError(err.value.decode())
        return out

    def close(self):
        if self.slot:
            self.lib.eg2cref_slot_free(self.slot)
            self.slot = None
        if self.handle:
            self.lib.eg2cref_close(self.handle)
            self.handle = None


class EngineLink:
    """The reference's own engine (engine.c, --backend kfd) linked with
    libeg2_b200.so (oracle/_ref/libeg2enginelink.so): its packed-wave call
    ei_engine_embed_tokens_batch reaches the B200 executor."""

    def __init__(self, model_path: str):
        if not os.path.exists(ENGINE_LINK_SO):
            raise FileNotFoundError(f"{ENGINE_LINK_SO} missing: run `make -C oracle engine_link`")
        self.lib = C.CDLL(ENGINE_LINK_SO)
        L = self.lib
        L.eg2link_open.restype = C.c_void_p
        L.eg2link_open.argtypes = [C.c_char_p]
        L.eg2link_backend.restype = C.c_char_p
        L.eg2link_backend.argtypes = [C.c_void_p]
        L.eg2link_embed_batch.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_char_p,
                                          C.c_size_t]
        L.eg2link_close.argtypes = [C.c_void_p]
        self.handle = L.eg2link_open(model_path.encode())

    @property
    def backend(self) -> str:
        return self.lib.eg2link_backend(self.handle).decode()

    def embed(self, ids, offsets):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        offsets = np.ascontiguousarray(offsets, dtype=np.uint64)
        batch = len(offsets) - 1
        out = np.zeros((batch, 768), np.float32)
        err = C.create_string_buffer(512)
        if not self.lib.eg2link_embed_batch(self.handle, _ptr(ids), _ptr(offsets), batch, _ptr(out), err, 512):
            raise RuntimeError(err.value.decode())
        return out

    def close(self):
        if self.handle:
            self.lib.eg2link_close(self.handle)
            self.handle = None


class Port:
    """The C restatement oracle/eg2_oracle.c (scalar tier)."""

    ROUND_SCALAR, ROUND_X86 = 0, 1

    def __init__(self):
        if not os.path.exists(PORT_SO):
            build(ref=False)
        self.lib = C.CDLL(PORT_SO)
        L = self.lib
        vp, i, f = C.c_void_p, C.c_int, C.c_float
        L.eg2o_fp32_to_fp16.argtypes = [f]
        L.eg2o_fp32_to_fp16.restype = C.c_uint16
        L.eg2o_fp16_to_fp32.argtypes = [C.c_uint16]
        L.eg2o_fp16_to_fp32.restype = f
        L.eg2o_quantize.argtypes = [vp, vp, vp, i, i]
        L.eg2o_gelu_mul.argtypes = [vp, vp, i, i]
        L.eg2o_gemm_q8.argtypes = [vp, vp, vp, vp, i, i, i, vp]
        L.eg2o_gemm_q8_blockdots.argtypes = [vp, vp, i, i, i, vp]
        L.eg2o_gemm_bf16.argtypes = [vp, vp, i, i, i, vp]
        L.eg2o_rms_row.argtypes = [vp, i, vp]
        L.eg2o_rope_tables.argtypes = [i, vp, vp]
        L.eg2o_attention.argtypes = [vp, vp, vp, vp, vp, i, i, i, i, vp]
        L.eg2o_embed_batch.argtypes = [vp, vp, vp, C.c_size_t, vp, i, i, vp]
        L.eg2o_embed_batch_inputs.argtypes = [vp, vp, vp, C.c_size_t, vp, i, i]
        L.eg2o_embed_trace.argtypes = [vp, vp, vp, C.c_size_t, vp, i, i, vp, vp]
        L.eg2o_layer.argtypes = [vp, i, vp, vp, vp, C.c_size_t, i, i]
        L.eg2o_set_variant.argtypes = [i, i]
        L.eg2o_set_order.argtypes = [i]

    def quantize(self, x, mode=ROUND_X86):
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        q = np.zeros(x.size, np.int8)
        d = np.zeros(x.size // 32, np.uint16)
        self.lib.eg2o_quantize(_ptr(x), _ptr(q), _ptr(d), x.size, mode)
        return q, d

    def gelu_mul(self, g, u, mode=1):
        g = np.array(g, dtype=np.float32, copy=True).ravel()
        u = np.ascontiguousarray(u, dtype=np.float32).ravel() if u is not None else None  # kept alive
        self.lib.eg2o_gelu_mul(_ptr(g), _ptr(u) if u is not None else None, g.size, mode)
        return g

    def gemm_q8(self, wq, wd, xq, xd):
        m, k = wq.shape
        n = xq.shape[0]
        y = np.zeros((n, m), np.float32)
        wq, wd, xq, xd = (np.ascontiguousarray(a) for a in (wq, wd, xq, xd))
        self.lib.eg2o_gemm_q8(_ptr(wq), _ptr(wd), _ptr(xq), _ptr(xd), n, k, m, _ptr(y))
        return y

    def gemm_q8_blockdots(self, wq, xq):
        m, k = wq.shape
        n = xq.shape[0]
        D = np.zeros((n, m, k // 32), np.int32)
        wq, xq = np.ascontiguousarray(wq), np.ascontiguousarray(xq)
        self.lib.eg2o_gemm_q8_blockdots(_ptr(wq), _ptr(xq), n, k, m, _ptr(D))
        return D

    def gemm_bf16(self, w_bits, x):
        m, k = w_bits.shape
        n = x.shape[0]
        y = np.zeros((n, m), np.float32)
        w_bits, x = np.ascontiguousarray(w_bits), np.ascontiguousarray(x, dtype=np.float32)
        self.lib.eg2o_gemm_bf16(_ptr(w_bits), _ptr(x), n, k, m, _ptr(y))
        return y

    def rms_rows(self, x, w):
        x = np.array(x, dtype=np.float32, copy=True)
        d = x.shape[-1]
        rows = x.reshape(-1, d)
        w = np.ascontiguousarray(w, dtype=np.float32) if w is not None else None  # kept alive
        wp = _ptr(w) if w is not None else None
        for r in range(rows.shape[0]):
            self.lib.eg2o_rms_row(C.c_void_p(rows[r:].ctypes.data), d, wp)
        return x

    def rope_tables(self, d):
        c = np.zeros((8192, d // 2), np.float32)
        s = np.zeros((8192, d // 2), np.float32)
        self.lib.eg2o_rope_tables(d, _ptr(c), _ptr(s))
        return c, s

    def attention(self, q, k, v, lo, hi, kv, d, window):
        n = q.shape[0]
        a = np.zeros((n, 4 * d), np.float32)
        q, k, v = (np.ascontiguousarray(t, dtype=np.float32) for t in (q, k, v))
        lo, hi = np.ascontiguousarray(lo, dtype=np.uint32), np.ascontiguousarray(hi, dtype=np.uint32)
        self.lib.eg2o_attention(_ptr(q), _ptr(k), _ptr(v), _ptr(lo), _ptr(hi), n, kv, d, window, _ptr(a))
        return a

    def embed(self, model: Gguf, ids, offsets, quant_mode=ROUND_SCALAR, gelu_mode=0, dump_layers=False):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        offsets = np.ascontiguousarray(offsets, dtype=np.uint64)
        batch = len(offsets) - 1
        n = int(offsets[-1])
        out = np.zeros((batch, 768), np.float32)
        xl = np.zeros((25, n, 512), np.float32) if dump_layers else None
        rc = self.lib.eg2o_embed_batch(model.pointer_table(), _ptr(ids), _ptr(offsets), batch, _ptr(out),
                                       quant_mode, gelu_mode, _ptr(xl) if dump_layers else None)
        if rc:
            raise RuntimeError("oracle rejected the wave")
        return (out, xl) if dump_layers else out

    def trace(self, model: Gguf, ids, offsets, quant_mode=ROUND_X86, gelu_mode=1):
        """The graph with its intermediate state: (embeddings [batch][768],
        residual stream entering each layer and after the last [25][n][512],
        per-layer embeddings [n][24][512])."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        offsets = np.ascontiguousarray(offsets, dtype=np.uint64)
        batch = len(offsets) - 1
        n = int(offsets[-1])
        out = np.zeros((batch, 768), np.float32)
        xl = np.zeros((25, n, 512), np.float32)
        ple = np.zeros((n, 24, 512), np.float32)
        if self.lib.eg2o_embed_trace(model.pointer_table(), _ptr(ids), _ptr(offsets), batch, _ptr(out),
                                     quant_mode, gelu_mode, _ptr(xl), _ptr(ple)):
            raise RuntimeError("oracle rejected the wave")
        return out, xl, ple

    def layer(self, model: Gguf, l, x, ple, offsets, quant_mode=ROUND_X86, gelu_mode=1):
        """One layer on the residual stream x [n][512] with the wave's per-layer
        embeddings ple [n][24][512]; returns the new x."""
        x = np.array(x, dtype=np.float32, copy=True).reshape(-1, 512)
        ple = np.ascontiguousarray(ple, dtype=np.float32)
        offsets = np.ascontiguousarray(offsets, dtype=np.uint64)
        assert ple.size == x.shape[0] * 24 * 512
        if self.lib.eg2o_layer(model.pointer_table(), l, _ptr(x), _ptr(ple), _ptr(offsets), len(offsets) - 1,
                               quant_mode, gelu_mode):
            raise RuntimeError("oracle rejected the layer")
        return x

    ORDER_SCALAR, ORDER_VNNI512 = 0, 1

    def set_order(self, order):
        """Float order of the restatement: ORDER_SCALAR (the scalar loops) or
        ORDER_VNNI512 (the reference's default tier on an AVX-512 VNNI host)."""
        self.lib.eg2o_set_order(int(order))

    def set_variant(self, gemm_descending=False, attention_fp16=False):
        """Perturb the restatement (tests of the float-order floor only)."""
        self.lib.eg2o_set_variant(int(gemm_descending), int(attention_fp16))

    def embed_inputs(self, model: Gguf, inputs, offsets, quant_mode=ROUND_SCALAR, gelu_mode=0):
        """The graph from 512-wide input rows (media soft tokens) instead of ids."""
        inputs = np.ascontiguousarray(inputs, dtype=np.float32).reshape(-1, 512)
        offsets = np.ascontiguousarray(offsets, dtype=np.uint64)
        batch = len(offsets) - 1
        assert inputs.shape[0] == int(offsets[-1])
        out = np.zeros((batch, 768), np.float32)
        rc = self.lib.eg2o_embed_batch_inputs(model.pointer_table(), _ptr(inputs), _ptr(offsets), batch,
                                              _ptr(out), quant_mode, gelu_mode)
        if rc:
            raise RuntimeError("oracle rejected the wave")
        return out
