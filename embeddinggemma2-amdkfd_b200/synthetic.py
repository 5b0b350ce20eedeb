"""Seeded synthetic EmbeddingGemma 2 GGUF files and packed token waves.

There is no network and no real checkpoint, so every run (tests, smoke, bench)
uses a random-init model with the reference's tensor names, shapes, types and
hyperparameters, written as a GGUF v3 file that the reference's own loader
accepts:

* hyperparameters and tensor table: vendor/embeddinggemma.c/src/gemma2.c:30-62
  (`ei_gemma2_validate`), GGUF layout: vendor/embeddinggemma.c/src/gguf.c:124-205;
* Q8_0 block = fp16 scale + 32 int8 (vendor/embeddinggemma.c/src/quants.h:13-19);
* every Q8_0 matrix: int8 uniform in [-127, 127], fp16 block scale
  |N(0, 1/sqrt(K))| * sqrt(3) / 127 with K the row length;
* `per_layer_model_proj.weight` is BF16 N(0, 1/sqrt(512)), as in the real file;
* norm weights fp32: ``norm="plus1"`` draws 1 + N(0, 0.1) (the real files bake
  the +1 in), ``norm="baseline"`` draws N(0, 0.1);
* `layer_output_scale`: one fp32 per layer, U[0.5, 1.0].

Token waves follow the reference's tokenizer convention: BOS=2 first and
EOS=1 last in every sequence, body ids uniform in [3, 262144).
"""
from __future__ import annotations

import hashlib
import os
import struct
import tempfile

import numpy as np

ARCH = "gemma-embedding2"
N_LAYER = 24
N_EMBD = 512
N_FF = 2048
N_OUT = 768
N_VOCAB = 262144
SLIDING_WINDOW = 1024
BOS, EOS = 2, 1

GGML_F32, GGML_F16, GGML_Q8_0, GGML_BF16 = 0, 1, 8, 30
GGUF_I32, GGUF_U32, GGUF_F32, GGUF_STRING, GGUF_ARRAY = 5, 4, 6, 8, 9
ALIGN = 32


def layer_dims(layer: int) -> tuple[int, int]:
    """(head_dim, kv_heads): every 6th layer is global (d=512, 1 KV head)."""
    d = 512 if layer % 6 == 5 else 256
    return d, 512 // d


def tensor_table():
    """[(name, type, ne0, ne1)] in the reference's naming (gemma2.c:39-61)."""
    t = [("token_embd.weight", GGML_Q8_0, N_EMBD, N_VOCAB),
         ("per_layer_model_proj.weight", GGML_BF16, N_EMBD, N_LAYER * N_EMBD),
         ("per_layer_proj_norm.weight", GGML_F32, N_EMBD, 1)]
    for l in range(N_LAYER):
        d, _ = layer_dims(l)
        p = f"blk.{l}."
        t += [(p + "attn_norm.weight", GGML_F32, 512, 1),
              (p + "attn_q.weight", GGML_Q8_0, 512, 4 * d),
              (p + "attn_k.weight", GGML_Q8_0, 512, 512),
              (p + "attn_v.weight", GGML_Q8_0, 512, 512),
              (p + "attn_output.weight", GGML_Q8_0, 4 * d, 512),
              (p + "attn_q_norm.weight", GGML_F32, d, 1),
              (p + "attn_k_norm.weight", GGML_F32, d, 1),
              (p + "post_attention_norm.weight", GGML_F32, 512, 1),
              (p + "ffn_norm.weight", GGML_F32, 512, 1),
              (p + "ffn_up.weight", GGML_Q8_0, 512, 2048),
              (p + "ffn_gate.weight", GGML_Q8_0, 512, 2048),
              (p + "ffn_down.weight", GGML_Q8_0, 2048, 512),
              (p + "post_ffw_norm.weight", GGML_F32, 512, 1),
              (p + "inp_gate.weight", GGML_Q8_0, 512, 512),
              (p + "proj.weight", GGML_Q8_0, 512, 512),
              (p + "post_norm.weight", GGML_F32, 512, 1),
              (p + "layer_output_scale.weight", GGML_F32, 1, 1)]
    t += [("output_norm.weight", GGML_F32, 512, 1),
          ("output.weight", GGML_Q8_0, 512, N_OUT)]
    return t


def _nbytes(typ: int, ne0: int, ne1: int) -> int:
    n = ne0 * ne1
    return {GGML_F32: 4 * n, GGML_F16: 2 * n, GGML_BF16: 2 * n, GGML_Q8_0: n // 32 * 34}[typ]


def _q8_blocks(rng: np.random.Generator, ne0: int, ne1: int) -> bytes:
    nb = ne0 * ne1 // 32
    q = rng.integers(-127, 128, size=(nb, 32), dtype=np.int8)
    d = (np.abs(rng.standard_normal(nb, dtype=np.float32)) / np.float32(np.sqrt(ne0))
         * np.float32(np.sqrt(3.0) / 127.0)).astype(np.float16)
    blk = np.empty((nb, 34), dtype=np.uint8)
    blk[:, :2] = d.view(np.uint8).reshape(nb, 2)
    blk[:, 2:] = q.view(np.uint8)
    return blk.tobytes()


def _norm(rng: np.random.Generator, n: int, mode: str) -> np.ndarray:
    w = rng.normal(0.0, 0.1, size=n).astype(np.float32)
    return (w + np.float32(1.0)) if mode == "plus1" else w


def _tensor_bytes(rng, name, typ, ne0, ne1, norm):
    if typ == GGML_Q8_0:
        return _q8_blocks(rng, ne0, ne1)
    if typ == GGML_BF16:
        f = rng.normal(0.0, 1.0 / np.sqrt(ne0), size=ne0 * ne1).astype(np.float32)
        return (f.view(np.uint32) >> 16).astype(np.uint16).tobytes()
    if name.endswith("layer_output_scale.weight"):
        return rng.uniform(0.5, 1.0, size=1).astype(np.float32).tobytes()
    return _norm(rng, ne0 * ne1, norm).tobytes()


def _kv_string(key: str, val: str) -> bytes:
    k, v = key.encode(), val.encode()
    return struct.pack("<Q", len(k)) + k + struct.pack("<I", GGUF_STRING) + struct.pack("<Q", len(v)) + v


def _kv_u32(key: str, val: int) -> bytes:
    k = key.encode()
    return struct.pack("<Q", len(k)) + k + struct.pack("<II", GGUF_U32, val)


def _kv_array(key: str, elem_type: int, payload: bytes, n: int) -> bytes:
    k = key.encode()
    return struct.pack("<Q", len(k)) + k + struct.pack("<IIQ", GGUF_ARRAY, elem_type, n) + payload


def _tokenizer_kvs() -> list[bytes]:
    """A placeholder tokenizer section for the reference's model loader
    (vendor/embeddinggemma.c/src/model.c:46-52,111-120; tokenizer.c:205-266):
    262144 pieces -- <pad>, <eos>, <bos>, <unk>, the 256 byte-fallback pieces
    <0xXX>, then filler pieces -- with zero scores, the usual token types and
    one merge.  It lets the reference's engine load the seeded model; text
    tokenization with it is not meaningful (callers pass token ids)."""
    pieces = ["<pad>", "<eos>", "<bos>", "<unk>"] + [f"<0x{b:02X}>" for b in range(256)]
    pieces += [f"\u2581t{i}" for i in range(N_VOCAB - len(pieces))]
    types = np.ones(N_VOCAB, np.int32)
    types[[0, 1, 2]] = 3   # control
    types[3] = 2           # unknown
    types[4:260] = 6       # byte
    enc = [x.encode() for x in pieces]
    tok = b"".join(struct.pack("<Q", len(e)) + e for e in enc)
    merge = "\u2581 t".encode()
    return [_kv_string("tokenizer.ggml.model", "gemma4"),
            _kv_array("tokenizer.ggml.tokens", GGUF_STRING, tok, N_VOCAB),
            _kv_array("tokenizer.ggml.scores", GGUF_F32, np.zeros(N_VOCAB, np.float32).tobytes(), N_VOCAB),
            _kv_array("tokenizer.ggml.token_type", GGUF_I32, types.tobytes(), N_VOCAB),
            _kv_array("tokenizer.ggml.merges", GGUF_STRING, struct.pack("<Q", len(merge)) + merge, 1)]


def write_gguf(path: str, seed: int = 1234, norm: str = "plus1", tokenizer: bool = False) -> str:
    """Write the seeded model to `path` and return the sha256 of the file.
    With tokenizer=True the file also carries a placeholder tokenizer section
    (same tensors and values), which the reference's engine loader requires."""
    if norm not in ("plus1", "baseline"):
        raise ValueError("norm must be 'plus1' or 'baseline'")
    table = tensor_table()
    kvs = [_kv_string("general.architecture", ARCH),
           _kv_u32(f"{ARCH}.block_count", N_LAYER),
           _kv_u32(f"{ARCH}.embedding_length", N_EMBD),
           _kv_u32(f"{ARCH}.feed_forward_length", N_FF),
           _kv_u32(f"{ARCH}.embedding_length_out", N_OUT),
           _kv_u32(f"{ARCH}.attention.sliding_window", SLIDING_WINDOW),
           _kv_u32("general.alignment", ALIGN)]
    if tokenizer:
        kvs += _tokenizer_kvs()
    infos, offset = [], 0
    for name, typ, ne0, ne1 in table:
        nm = name.encode()
        dims = [ne0] if ne1 == 1 else [ne0, ne1]
        infos.append(struct.pack("<Q", len(nm)) + nm + struct.pack("<I", len(dims))
                     + b"".join(struct.pack("<Q", x) for x in dims)
                     + struct.pack("<IQ", typ, offset))
        offset += (_nbytes(typ, ne0, ne1) + ALIGN - 1) // ALIGN * ALIGN
    head = b"GGUF" + struct.pack("<IQQ", 3, len(table), len(kvs)) + b"".join(kvs) + b"".join(infos)
    pad = (-len(head)) % ALIGN
    rng = np.random.Generator(np.random.PCG64(seed))
    h = hashlib.sha256()
    tmp = f"{path}.{os.getpid()}.part"  # one writer per process; os.replace is atomic
    with open(tmp, "wb") as f:
        for chunk in (head, b"\0" * pad):
            f.write(chunk)
            h.update(chunk)
        for name, typ, ne0, ne1 in table:
            data = _tensor_bytes(rng, name, typ, ne0, ne1, norm)
            data += b"\0" * ((-len(data)) % ALIGN)
            f.write(data)
            h.update(data)
    os.replace(tmp, path)
    return h.hexdigest()


def model_path(seed: int = 1234, norm: str = "plus1", cache_dir: str | None = None, tokenizer: bool = False) -> str:
    """Path of the cached seeded model, written on first use (~151 MB)."""
    cache_dir = cache_dir or os.environ.get("EG2_MODEL_CACHE") or os.path.join(
        tempfile.gettempdir(), "eg2_b200_models")
    os.makedirs(cache_dir, exist_ok=True)
    path = os.path.join(cache_dir, f"eg2-synth-s{seed}-{norm}{'-tok' if tokenizer else ''}.gguf")
    if not os.path.exists(path):
        write_gguf(path, seed, norm, tokenizer)
    return path


def wave(lengths, seed: int = 7, bos_eos: bool = True):
    """Packed token ids (int32) and offsets (uint64, batch+1) for body lengths.

    With ``bos_eos`` each sequence is BOS + body + EOS, so its packed length is
    body + 2 (the reference tokenizer adds both; the empty text is [2, 1])."""
    rng = np.random.Generator(np.random.PCG64(seed))
    ids, offsets = [], [0]
    for n in lengths:
        body = rng.integers(3, N_VOCAB, size=int(n), dtype=np.int64).astype(np.int32)
        seq = np.concatenate([[BOS], body, [EOS]]).astype(np.int32) if bos_eos else body
        ids.append(seq)
        offsets.append(offsets[-1] + len(seq))
    return np.concatenate(ids).astype(np.int32), np.asarray(offsets, dtype=np.uint64)


# The BASELINE configurations restated in the real model's terms.
CONFIG0_BODIES = (8, 17, 33, 64)          # 4 sequences -> 130 packed tokens
CONFIG1_BODIES = (126,) * 16              # 16 x 128 = 2048 packed tokens
CONFIG2_BODIES = (2046,)                  # 1 x 2048 packed tokens


def mixed_load(requests: int = 256, texts: int = 16, seed: int = 11):
    """Config 3: per-text body lengths lognormal(median 48, sigma 1) clipped to
    [4, 2048] packed tokens, dims uniform in {128, 256, 512, 768} per request."""
    rng = np.random.Generator(np.random.PCG64(seed))
    lens = np.clip(np.round(rng.lognormal(np.log(48.0), 1.0, size=(requests, texts))), 4, 2048)
    dims = rng.choice(np.array([128, 256, 512, 768]), size=requests)
    return (lens.astype(np.int64) - 2), dims
