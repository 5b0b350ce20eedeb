"""Python mirror of the executor C ABI (include/eg2_executor.h).

Same names, argument meaning and error behaviour as the reference's
`ei_gemma2_kfd_create / _free / _batch` (src/gemma2_kfd.h:7-10): host arrays
in, L2-normalised batch x 768 float32 embeddings out, failures raised as
`ExecutorError("KFD: ...")` carrying the library's message.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib

EMBED_DIM = 768
MAX_TOKENS = 2048
WIDE_MAX_TOKENS = 8192  # EG2_B200_WAVE_8192
VOCAB = 262144


EG2_B200_EXACT, EG2_B200_SCALAR_TIER, EG2_B200_WAVE_8192, EG2_B200_VNNI512_TIER = 1, 2, 4, 8  # include/eg2_executor.h


class ExecutorError(RuntimeError):
    pass


def _err():
    return C.create_string_buffer(512)


def _wave(ids, offsets):
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    offsets = np.ascontiguousarray(offsets, dtype=np.uint64)
    return ids, offsets, len(offsets) - 1


def _rows(rows, offsets):
    rows = np.ascontiguousarray(rows, dtype=np.float32)
    offsets = np.ascontiguousarray(offsets, dtype=np.uint64)
    if rows.size % 512:
        raise ExecutorError("input rows must be 512 wide")
    rows = rows.reshape(-1, 512)
    if len(offsets) and rows.shape[0] != int(offsets[-1]):
        raise ExecutorError("input rows do not match offsets")
    return rows, offsets, len(offsets) - 1


def validate(ids, offsets) -> None:
    """The reference's host-side wave checks (gemma2_kfd.cpp:270-278), no GPU needed."""
    ids, offsets, batch = _wave(ids, offsets)
    err = _err()
    if not _lib.load().eg2_b200_validate(ids.ctypes.data if ids.size else None,
                                         offsets.ctypes.data if offsets.size else None, max(batch, 0), err,
                                         len(err)):
        raise ExecutorError(err.value.decode())


def validate_rows(rows, offsets) -> None:
    """The host-side checks of a soft-token wave (offsets as for ids), no GPU needed."""
    rows = np.ascontiguousarray(rows, dtype=np.float32)
    offsets = np.ascontiguousarray(offsets, dtype=np.uint64)
    batch = len(offsets) - 1
    err = _err()
    if not _lib.load().eg2_b200_validate_rows(rows.ctypes.data if rows.size else None,
                                              offsets.ctypes.data if offsets.size else None, max(batch, 0), err,
                                              len(err)):
        raise ExecutorError(err.value.decode())


class GGUFModel:
    """A GGUF file mapped by the library's own loader into an `ei_gguf`."""

    def __init__(self, path: str):
        lib = _lib.load()
        self._buf = C.create_string_buffer(lib.eg2_gguf_struct_size())
        err = _err()
        if not lib.eg2_gguf_open(self._buf, path.encode(), err, len(err)):
            self._buf = None
            raise ExecutorError(err.value.decode())
        self.path = path

    @property
    def handle(self):
        return C.cast(self._buf, C.c_void_p)

    def close(self):
        if getattr(self, "_buf", None) is not None:
            _lib.load().eg2_gguf_close(self._buf)
            self._buf = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Gemma2Executor:
    """One packed-wave executor on one B200 (ei_gemma2_kfd_create_on)."""

    def __init__(self, model: GGUFModel, device: int | None = None, exact: bool = False, tier: str = "x86",
                 max_tokens: int = MAX_TOKENS):
        """exact=True: parity mode (eg2_b200_create with EG2_B200_EXACT), every
        operation in the reference CPU graph's own float order; tier="scalar"
        adds the scalar CPU tier's quantizer rounding and GELU
        (EG2_B200_SCALAR_TIER), so the wave reproduces that tier;
        tier="vnni512" the float orders, quantizer and GELU of its default tier
        on an AVX-512 VNNI host (EG2_B200_VNNI512_TIER), so the wave reproduces
        that one.
        max_tokens=8192: waves up to the reference CPU graph's limit
        (EG2_B200_WAVE_8192; fast path only)."""
        lib = _lib.load()
        self.model = model  # borrowed by the context: keep it alive
        err = _err()
        if tier not in ("x86", "scalar", "vnni512"):
            raise ValueError("tier must be 'x86', 'scalar' or 'vnni512'")
        if tier == "vnni512" and not exact:
            raise ValueError("tier 'vnni512' is a parity-mode tier (exact=True)")
        if max_tokens not in (MAX_TOKENS, WIDE_MAX_TOKENS):
            raise ValueError(f"max_tokens must be {MAX_TOKENS} or {WIDE_MAX_TOKENS}")
        if exact or max_tokens == WIDE_MAX_TOKENS:
            flags = (EG2_B200_EXACT if exact else 0) | (EG2_B200_SCALAR_TIER if exact and tier == "scalar" else 0)
            flags |= EG2_B200_VNNI512_TIER if exact and tier == "vnni512" else 0
            flags |= EG2_B200_WAVE_8192 if max_tokens == WIDE_MAX_TOKENS else 0
            ctx = lib.eg2_b200_create(model.handle, 0 if device is None else int(device), flags, err, len(err))
        elif device is None:
            ctx = lib.ei_gemma2_kfd_create(model.handle, err, len(err))
        else:
            ctx = lib.ei_gemma2_kfd_create_on(model.handle, int(device), err, len(err))
        if not ctx:
            raise ExecutorError(err.value.decode())
        self.ctx = ctx
        self.lib = lib
        self._staged_batch = 0
        self._slot_batch = {}

    def batch(self, ids, offsets) -> np.ndarray:
        """Embed one packed wave: ids int32[n], offsets (batch+1) with offsets[0]=0."""
        ids, offsets, batch = _wave(ids, offsets)
        out = np.zeros((max(batch, 1), EMBED_DIM), np.float32)
        err = _err()
        ok = self.lib.ei_gemma2_kfd_batch(self.ctx, ids.ctypes.data if ids.size else None,
                                          offsets.ctypes.data if offsets.size else None, max(batch, 0),
                                          out.ctypes.data, err, len(err))
        if not ok:
            raise ExecutorError(err.value.decode())
        return out[:batch]

    # pipelined form: two slots, collect a slot before submitting to it again
    def submit(self, ids, offsets) -> int:
        """Stage and enqueue one packed wave; returns the slot to collect."""
        ids, offsets, batch = _wave(ids, offsets)
        err = _err()
        slot = self.lib.eg2_b200_submit(self.ctx, ids.ctypes.data if ids.size else None,
                                        offsets.ctypes.data if offsets.size else None, max(batch, 0), err, len(err))
        if slot < 0:
            raise ExecutorError(err.value.decode())
        self._slot_batch[slot] = batch
        return slot

    def collect(self, slot: int) -> np.ndarray:
        """Wait for a submitted wave and return its embeddings."""
        batch = self._slot_batch.get(slot, 0)
        out = np.zeros((max(batch, 1), EMBED_DIM), np.float32)
        err = _err()
        if not self.lib.eg2_b200_collect(self.ctx, slot, out.ctypes.data, err, len(err)):
            raise ExecutorError(err.value.decode())
        return out[:batch]

    # media soft-token waves: 512-wide input rows instead of token ids
    def batch_rows(self, rows, offsets) -> np.ndarray:
        """Embed one packed wave given as rows float32[n][512] (the reference CPU
        graph's ids == NULL form, gemma2_fast.c:940-941)."""
        rows, offsets, batch = _rows(rows, offsets)
        out = np.zeros((max(batch, 1), EMBED_DIM), np.float32)
        err = _err()
        if not self.lib.eg2_b200_batch_rows(self.ctx, rows.ctypes.data if rows.size else None,
                                            offsets.ctypes.data if offsets.size else None, max(batch, 0),
                                            out.ctypes.data, err, len(err)):
            raise ExecutorError(err.value.decode())
        return out[:batch]

    def submit_rows(self, rows, offsets) -> int:
        rows, offsets, batch = _rows(rows, offsets)
        err = _err()
        slot = self.lib.eg2_b200_submit_rows(self.ctx, rows.ctypes.data if rows.size else None,
                                             offsets.ctypes.data if offsets.size else None, max(batch, 0), err,
                                             len(err))
        if slot < 0:
            raise ExecutorError(err.value.decode())
        self._slot_batch[slot] = batch
        return slot

    def stage_rows(self, rows, offsets):
        rows, offsets, batch = _rows(rows, offsets)
        err = _err()
        if not self.lib.eg2_b200_stage_rows(self.ctx, rows.ctypes.data, offsets.ctypes.data, batch, err, len(err)):
            raise ExecutorError(err.value.decode())
        self._staged_batch = batch

    # split form, for device-resident timing
    def stage(self, ids, offsets):
        ids, offsets, batch = _wave(ids, offsets)
        err = _err()
        if not self.lib.eg2_b200_stage(self.ctx, ids.ctypes.data, offsets.ctypes.data, batch, err, len(err)):
            raise ExecutorError(err.value.decode())
        self._staged_batch = batch

    def launch(self, repeats: int = 1):
        err = _err()
        if not self.lib.eg2_b200_launch(self.ctx, int(repeats), err, len(err)):
            raise ExecutorError(err.value.decode())

    def finish(self) -> np.ndarray:
        out = np.zeros((max(self._staged_batch, 1), EMBED_DIM), np.float32)
        err = _err()
        if not self.lib.eg2_b200_finish(self.ctx, out.ctypes.data, err, len(err)):
            raise ExecutorError(err.value.decode())
        return out[:self._staged_batch]

    def forward_layers(self, x, ple, offsets, first: int, last: int) -> np.ndarray:
        """Layers [first, last) on a given residual stream x [n][512] with the
        wave's per-layer embeddings ple [n][24][512] (None: projected from x,
        the embedding rows); returns the residual stream after layer last - 1
        (eg2_b200_forward_layers)."""
        x, offsets, batch = _rows(x, offsets)
        n = x.shape[0]
        if ple is not None:
            ple = np.ascontiguousarray(ple, dtype=np.float32)
            if ple.size != n * 24 * 512:
                raise ExecutorError("per-layer embeddings must be [n][24][512]")
        out = np.zeros((max(n, 1), 512), np.float32)
        err = _err()
        if not self.lib.eg2_b200_forward_layers(self.ctx, x.ctypes.data if x.size else None,
                                                ple.ctypes.data if ple is not None else None,
                                                offsets.ctypes.data if offsets.size else None, max(batch, 0),
                                                int(first), int(last), out.ctypes.data, err, len(err)):
            raise ExecutorError(err.value.decode())
        return out[:n]

    def prepare(self, max_tokens: int) -> int:
        """Capture the graphs of every wave shape up to max_tokens on both lanes
        now (eg2_b200_prepare); returns the number of graphs held."""
        err = _err()
        n = self.lib.eg2_b200_prepare(self.ctx, int(max_tokens), err, len(err))
        if n < 0:
            raise ExecutorError(err.value.decode())
        return n

    @property
    def stream(self) -> int:
        return int(self.lib.eg2_b200_stream(self.ctx) or 0)

    @property
    def kernels_per_wave(self) -> int:
        return int(self.lib.eg2_b200_kernels_per_wave(self.ctx))

    @property
    def device(self) -> int:
        return int(self.lib.eg2_b200_device(self.ctx))

    def profile(self) -> dict:
        """Milliseconds per kernel group of one eager run of the staged wave."""
        names = (C.c_char * 32 * 64)()
        ms = (C.c_double * 64)()
        k = self.lib.eg2_b200_profile(self.ctx, names, ms, 64)
        if k < 0:
            raise ExecutorError("KFD: profile failed")
        return {bytes(names[i]).split(b"\0", 1)[0].decode(): float(ms[i]) for i in range(k)}

    def close(self):
        if getattr(self, "ctx", None):
            self.lib.ei_gemma2_kfd_free(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def normalize_prefix(embedding: np.ndarray, dimensions: int) -> np.ndarray:
    """Matryoshka truncation as the server applies it
    (vendor/embeddinggemma.c/src/kernels.c:398-407, server.c:1133): keep the
    first `dimensions` in {128, 256, 512, 768} and L2-renormalise when shorter,
    in the reference's float order (eg2_b200_normalize_prefix, host code)."""
    if dimensions not in (128, 256, 512, 768):
        raise ValueError("dimensions must be one of 128, 256, 512, 768")
    e = np.array(embedding, dtype=np.float32, copy=True)
    if e.shape[-1] != EMBED_DIM:
        raise ValueError("embeddings must be 768 wide")
    lib = _lib.load()
    flat = np.ascontiguousarray(e.reshape(-1, EMBED_DIM))
    for row in flat:
        lib.eg2_b200_normalize_prefix(row.ctypes.data, dimensions)
    return np.ascontiguousarray(flat.reshape(e.shape)[..., :dimensions])
