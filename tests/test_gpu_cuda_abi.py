"""The reference's CUDA executor ABI (vendor/embeddinggemma.c/src/gemma2_cuda.h:
13-33) as libeg2_b200.so exports it (include/gemma2_cuda.h), called through
ctypes the way the reference's engine calls it (engine.c:1199-1220, 1298-1300):
a context per device, clones as pipeline slots, packed batches of more than
8192 tokens split at sequence boundaries (gemma2_cuda.cu:1451-1468), one
sequence of input rows, the media towers refused with a message."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda_abi(eg2, model_baseline):
    lib = eg2._lib.load()
    m = eg2.GGUFModel(model_baseline)
    err = C.create_string_buffer(512)
    ctx = lib.ei_gemma2_cuda_create_on(m.handle, 0, err, len(err))
    assert ctx, err.value
    yield lib, ctx, m
    lib.ei_gemma2_cuda_free(ctx)
    m.close()


def _batch(lib, ctx, ids, off):
    ids = np.ascontiguousarray(ids, np.int32)
    off = np.ascontiguousarray(off, np.uint64)
    out = np.zeros((len(off) - 1, 768), np.float32)
    err = C.create_string_buffer(512)
    ok = lib.ei_gemma2_cuda_batch(ctx, ids.ctypes.data, off.ctypes.data, len(off) - 1, out.ctypes.data, err, len(err))
    return ok, out, err.value.decode()


def test_device_and_errors(cuda_abi, eg2, model_baseline):
    lib, ctx, m = cuda_abi
    assert lib.ei_gemma2_cuda_device_count() >= 1
    assert lib.ei_gemma2_cuda_device(ctx) == 0
    err = C.create_string_buffer(512)
    assert not lib.ei_gemma2_cuda_create_on(m.handle, 999, err, len(err))
    assert "does not exist" in err.value.decode()
    ok, _, msg = _batch(lib, ctx, np.zeros(9000, np.int32), [0, 9000])
    assert not ok and msg == "EmbeddingGemma 2 accepts 1..8192 tokens per wave"
    assert not lib.ei_gemma2_cuda_vision(ctx, None, None, 4, 4, None, None, err, len(err))
    assert "image tower" in err.value.decode()
    assert not lib.ei_gemma2_cuda_audio(ctx, None, None, 4, None, None, err, len(err))
    assert "audio tower" in err.value.decode()


def test_batches_over_8192_tokens_split_and_clones_share_the_context(cuda_abi, eg2, syn, model_baseline):
    """Five 2046-body sequences (10240 tokens) come back as two waves' worth of
    embeddings equal, bit for bit, to each sequence alone; a clone returns the
    same, and freeing it leaves the parent working."""
    lib, ctx, m = cuda_abi
    ids, off = syn.wave((2046,) * 5, seed=71)
    ok, out, msg = _batch(lib, ctx, ids, off)
    assert ok, msg
    err = C.create_string_buffer(512)
    clone = lib.ei_gemma2_cuda_clone(ctx, True, err, len(err))
    assert clone, err.value
    for s in range(5):
        seq = ids[off[s]:off[s + 1]]
        ok, solo, msg = _batch(lib, clone, seq, [0, len(seq)])
        assert ok, msg
        np.testing.assert_array_equal(solo[0], out[s])
    lib.ei_gemma2_cuda_free(clone)
    ok, again, msg = _batch(lib, ctx, ids[:off[1]], off[:2])
    assert ok, msg
    np.testing.assert_array_equal(again[0], out[0])


def test_embed_inputs_equals_the_rows_batch(cuda_abi, eg2, model_baseline):
    lib, ctx, m = cuda_abi
    rows = np.random.Generator(np.random.PCG64(3)).standard_normal((37, 512)).astype(np.float32)
    out = np.zeros(768, np.float32)
    err = C.create_string_buffer(512)
    assert lib.ei_gemma2_cuda_embed_inputs(ctx, rows.ctypes.data, 37, out.ctypes.data, err, len(err)), err.value
    ex = eg2.Gemma2Executor(eg2.GGUFModel(model_baseline), 0)
    try:
        np.testing.assert_array_equal(out, ex.batch_rows(rows, np.array([0, 37], np.uint64))[0])
    finally:
        ex.close()
