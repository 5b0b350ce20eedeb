"""HTTP serving through the reference's own server (vendor/embeddinggemma.c/src/
server.c, inference_service.c and engine.c, built unchanged with
-DEI_ENABLE_KFD=1 against include/ into oracle/_ref/eg2server): with
`--backend kfd` its tokenizer, batcher and JSON layer sit in front of this
executor.  A request's embeddings must equal, bit for bit, what the executor
returns for the same tokens (tokenized by the reference engine's own tokenizer,
engine.c:1143) after the server's Matryoshka truncation (kernels.c:398-407,
eg2_b200_normalize_prefix) -- whatever waves the batcher packed them into."""
import ctypes as C
import http.client
import os
import sys

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

sys.path.insert(0, ROOT)
import bench  # noqa: E402  (the server start/stop and request helpers)

PORT = bench.free_port()


@pytest.fixture(scope="module")
def server(syn):
    if not os.path.exists(bench.SERVER_BIN):
        pytest.skip("oracle/_ref/eg2server not built (make -C oracle server)")
    proc = bench.start_server(bench.SERVER_BIN, syn.model_path(1234, "baseline", tokenizer=True), PORT, "kfd", 0)
    yield proc
    bench.stop_server(proc)


@pytest.fixture(scope="module")
def executor(eg2, model_baseline):
    m = eg2.GGUFModel(model_baseline)
    ex = eg2.Gemma2Executor(m, 0)
    yield ex
    ex.close()
    m.close()


@pytest.fixture(scope="module")
def tokenizer(syn):
    import oracle
    lib = C.CDLL(oracle.ENGINE_LINK_SO)
    lib.eg2link_open_cpu.restype = C.c_void_p
    lib.eg2link_open_cpu.argtypes = [C.c_char_p]
    lib.eg2link_tokenize.restype = C.c_size_t
    lib.eg2link_tokenize.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t, C.c_void_p, C.c_size_t]
    lib.eg2link_close.argtypes = [C.c_void_p]
    h = lib.eg2link_open_cpu(syn.model_path(1234, "baseline", tokenizer=True).encode())

    def tokenize(text):
        b = text.encode()
        ids = np.zeros(len(b) + 16, np.int32)
        n = lib.eg2link_tokenize(h, b, len(b), ids.ctypes.data, ids.size)
        return ids[:n].copy()
    yield tokenize
    lib.eg2link_close(h)


def test_http_embeddings_equal_the_executor(server, tokenizer, executor, eg2, syn):
    lens, dims = syn.mixed_load(8, 16, seed=3)
    texts = bench.http_texts(lens)
    conn = http.client.HTTPConnection("127.0.0.1", PORT, timeout=120)
    try:
        for r in range(len(texts)):
            d = int(dims[r])
            got = bench.http_embed(conn, texts[r], d)
            toks = [tokenizer(t) for t in texts[r]]
            assert [len(t) for t in toks] == [4 + len(t) for t in texts[r]]  # BOS + U+2581 + one token per byte
            for i, t in enumerate(toks):  # solo and packed waves embed a text bit-identically
                want = executor.batch(t, np.array([0, len(t)], np.uint64))[0]
                np.testing.assert_array_equal(got[i], eg2.normalize_prefix(want, d))
    finally:
        conn.close()


def test_http_over_long_request_is_a_client_error(server):
    """A text beyond the KFD executor's 2048 packed tokens is refused with a
    4xx, as the reference server maps executor errors (the server checks
    the KFD limit itself, server.c:2041)."""
    conn = http.client.HTTPConnection("127.0.0.1", PORT, timeout=120)
    try:
        body = b'{"input": ["' + b"a" * 2100 + b'"]}'
        conn.request("POST", "/api/embed", body=body, headers={"Content-Type": "application/json"})
        resp = conn.getresponse()
        resp.read()
        assert 400 <= resp.status < 500
    finally:
        conn.close()


PORT_CUDA = bench.free_port()


@pytest.fixture(scope="module")
def server_cuda(syn):
    """The reference server built for its CUDA backend (-DEI_ENABLE_CUDA)
    against include/gemma2_cuda.h: its engine drives this executor through the
    reference's CUDA executor ABI, with two pipeline slots (a context and one
    clone) and waves of up to 8192 tokens."""
    if not os.path.exists(bench.SERVER_CUDA_BIN):
        pytest.skip("oracle/_ref/eg2server_cuda not built (make -C oracle server)")
    proc = bench.start_server(bench.SERVER_CUDA_BIN, syn.model_path(1234, "baseline", tokenizer=True), PORT_CUDA,
                              "cuda", None, ("--cuda-devices", "0", "--pipeline-slots", "2", "--threads", "2"))
    yield proc
    bench.stop_server(proc)


def test_http_cuda_backend_equals_the_executor(server_cuda, tokenizer, executor, eg2, syn):
    """Requests sent concurrently over two connections, so that both pipeline
    slots carry waves; every embedding equals the executor's for its tokens."""
    import threading
    lens, dims = syn.mixed_load(12, 16, seed=4)
    texts = bench.http_texts(lens)
    got, errors = {}, []

    def client(rs):
        conn = http.client.HTTPConnection("127.0.0.1", PORT_CUDA, timeout=120)
        try:
            for r in rs:
                got[r] = bench.http_embed(conn, texts[r], int(dims[r]))
        except Exception as e:  # reported below
            errors.append(e)
        finally:
            conn.close()
    threads = [threading.Thread(target=client, args=(range(k, len(texts), 3),)) for k in range(3)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    for r in range(len(texts)):
        for i, t in enumerate(texts[r]):
            ids = tokenizer(t)
            want = executor.batch(ids, np.array([0, len(ids)], np.uint64))[0]
            np.testing.assert_array_equal(got[r][i], eg2.normalize_prefix(want, int(dims[r])))
