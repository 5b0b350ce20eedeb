"""End-to-end parity of the executor C ABI (ei_gemma2_kfd_create/_batch) on a
B200 against the reference's own CPU graph (golden fixtures made by
tests/golden/make_golden.py from oracle/_ref, and the live restatement).

Tolerance.  The reference's default CPU graph and its scalar tier run the
same math in different float orders and already disagree: on the BASELINE
model (norm weights N(0, 0.1)) they reach cosine 0.9982-0.9996 against each
other; one Q8_0 code that lands on the other side of a rounding boundary
changes the next GEMM's inputs, and 24 layers amplify it.  Where the
reference's two tiers are both at hand (config 0, the input-rows wave) the
bound is their own agreement minus MARGIN; elsewhere it is the value measured
on B200 minus a stated margin (each assertion gives both).  The per-layer,
teacher-forced tolerance is in test_gpu_layers.py; the per-operator tests
(test_gpu_ops.py) carry the bit-exact claims.
"""
import numpy as np
import pytest

from conftest import cosine, golden

pytestmark = pytest.mark.gpu
MARGIN = 0.0015  # measured worst: 0.0004 below the reference's own inter-tier agreement (config 0)


@pytest.fixture(scope="module")
def executor(eg2, model_baseline):
    m = eg2.GGUFModel(model_baseline)
    ex = eg2.Gemma2Executor(m, 0)
    yield ex
    ex.close()
    m.close()


def _floor(g):
    """The reference's own agreement between its x86 tiers on this wave."""
    return float(cosine(g["embed_scalar"], g["embed_best"]).min())


def test_config0_matches_reference(executor):
    g = golden("golden_baseline.npz")
    out = executor.batch(g["ids"], g["offsets"])
    assert out.shape == (4, 768)
    np.testing.assert_allclose(np.linalg.norm(out, axis=1), 1.0, atol=1e-5)
    floor = _floor(g)
    c_scalar = cosine(out, g["embed_scalar"])
    c_best = cosine(out, g["embed_best"])
    print("cos vs scalar tier", c_scalar, "vs best tier", c_best, "reference inter-tier", floor)
    assert c_scalar.min() >= floor - MARGIN
    assert c_best.min() >= floor - MARGIN


def test_long_and_two_wave_goldens(executor, eg2):
    g = golden("golden_long_baseline.npz")
    out = executor.batch(g["long_ids"], g["long_offsets"])
    c = float(cosine(out[0], g["long_embed"][0]))
    print("1x2048 cos", c)
    assert c >= 0.9999  # the north star; measured 0.99999
    for dims in (128, 256, 512):
        p = eg2.normalize_prefix(out[0], dims)
        assert abs(np.linalg.norm(p) - 1) < 1e-5
        cp = float(cosine(p, g[f"long_prefix_{dims}"]))
        print(f"1x2048 prefix {dims} cos", cp)
        assert cp >= 0.9999
    out2 = executor.batch(g["w2x128_ids"], g["w2x128_offsets"])
    c2 = cosine(out2, g["w2x128_embed"])
    print("2x128 cos", c2)
    assert c2.min() >= 0.9995  # measured 0.99980 - 0.0003


def test_submit_collect_pipeline_equals_batch(executor, syn):
    """Two waves in flight through the pipelined pair give exactly the batch
    call's embeddings; a slot cannot be submitted to again before collection."""
    waves = [syn.wave(lens, seed=s) for s, lens in enumerate([(40, 7, 300), (126,) * 16, (5,), (900, 900)])]
    expect = [executor.batch(ids, off) for ids, off in waves]
    s0 = executor.submit(*waves[0])
    s1 = executor.submit(*waves[1])
    assert s0 != s1
    with pytest.raises(Exception):
        executor.submit(*waves[2])  # slot s0 is still in flight
    np.testing.assert_array_equal(executor.collect(s0), expect[0])
    s2 = executor.submit(*waves[2])
    np.testing.assert_array_equal(executor.collect(s1), expect[1])
    s3 = executor.submit(*waves[3])
    np.testing.assert_array_equal(executor.collect(s2), expect[2])
    np.testing.assert_array_equal(executor.collect(s3), expect[3])
    with pytest.raises(Exception):
        executor.collect(s3)  # already collected


def test_concurrent_calls_equal_serial_calls(executor, syn):
    """ei_gemma2_kfd_batch from several host threads at once: the context runs
    two calls' waves on its two lanes concurrently (a third caller waits for
    a lane); every call returns exactly what it returns alone."""
    import threading
    waves = [syn.wave(lens, seed=50 + s) for s, lens in
             enumerate([(40, 7, 300), (126,) * 16, (5,), (900, 900), (64,) * 9, (2046,)])]
    expect = [executor.batch(ids, off) for ids, off in waves]
    got, errors = {}, []

    def caller(k):
        try:
            for r in range(3):
                i = (k + r) % len(waves)
                got[(k, r)] = (i, executor.batch(*waves[i]))
        except Exception as e:  # reported below, in the main thread
            errors.append(e)
    threads = [threading.Thread(target=caller, args=(k,)) for k in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    assert len(got) == 12
    for i, out in got.values():
        np.testing.assert_array_equal(out, expect[i])


def test_call_beside_submitted_wave_and_alternating_launches(executor, syn):
    """A synchronous call takes the lane a submitted wave leaves free; the
    split form's replays alternate over both lanes and end on the same
    embeddings as one replay."""
    w0, w1 = syn.wave((33, 300), seed=61), syn.wave((126,) * 16, seed=62)
    e0, e1 = executor.batch(*w0), executor.batch(*w1)
    s0 = executor.submit(*w0)
    np.testing.assert_array_equal(executor.batch(*w1), e1)
    np.testing.assert_array_equal(executor.collect(s0), e0)
    executor.stage(*w1)
    executor.launch(5)
    np.testing.assert_array_equal(executor.finish(), e1)
    executor.launch(1)
    np.testing.assert_array_equal(executor.finish(), e1)


def test_prepare_captures_every_wave_shape(eg2, model_baseline, syn):
    """eg2_b200_prepare captures the graphs of all 32 buckets of a 2048-token
    context on both lanes up front; later waves of any shape reuse them (the
    count stays 64) and give the same embeddings as a context that captured
    on first use."""
    import time
    m = eg2.GGUFModel(model_baseline)
    a, b = eg2.Gemma2Executor(m, 0), eg2.Gemma2Executor(m, 0)
    try:
        t0 = time.perf_counter()
        assert a.prepare(2048) == 64
        print(f"prepare(2048): {(time.perf_counter() - t0) * 1e3 / 64:.1f} ms per graph")
        for lens in [(5,), (40, 7, 300), (126,) * 16, (1000, 1000)]:
            ids, off = syn.wave(lens, seed=81)
            np.testing.assert_array_equal(a.batch(ids, off), b.batch(ids, off))
        assert a.prepare(2048) == 64
        assert a.prepare(100000) == 64  # clamped to the context's cap
    finally:
        a.close()
        b.close()
        m.close()


def test_packed_equals_solo_and_reorder(executor, syn):
    """tests/http_parity.py:62-69 (packed vs solo >= 0.99999, reorder
    invariance).  Every operation of a token depends only on its own sequence
    and is evaluated the same way wherever the sequence sits in the wave, so
    here the embeddings are bit-identical."""
    ids, off = syn.wave((8, 17, 33, 64, 200, 700), seed=31)
    packed = executor.batch(ids, off)
    for s in range(len(off) - 1):
        seq = ids[off[s]:off[s + 1]]
        solo = executor.batch(seq, np.array([0, len(seq)], np.uint64))[0]
        np.testing.assert_array_equal(solo, packed[s])
    order = [3, 0, 5, 4, 2, 1]
    seqs = [ids[off[s]:off[s + 1]] for s in order]
    ids2 = np.concatenate(seqs)
    off2 = np.concatenate([[0], np.cumsum([len(s) for s in seqs])]).astype(np.uint64)
    re = executor.batch(ids2, off2)
    for i, s in enumerate(order):
        np.testing.assert_array_equal(re[i], packed[s])


def test_repeatable_and_graph_reuse(executor, syn):
    ids, off = syn.wave((126,) * 16, seed=41)
    a = executor.batch(ids, off)
    b = executor.batch(ids, off)
    np.testing.assert_array_equal(a, b)
    assert executor.kernels_per_wave > 0


def test_errors_match_reference_messages(executor, eg2):
    """gemma2_kfd.cpp:271-278 messages; the context stays usable afterwards."""
    ok_ids = np.array([2, 5, 1], np.int32)
    cases = [
        (ok_ids, np.array([0, 0], np.uint64), "invalid KFD sequence offsets"),
        (ok_ids, np.array([1, 3], np.uint64), "1..2048 packed tokens"),
        (np.full(2049, 5, np.int32), np.array([0, 2049], np.uint64), "1..2048 packed tokens"),
        (np.array([2, 262144, 1], np.int32), np.array([0, 3], np.uint64), "token ID out of range"),
        (np.array([2, -1, 1], np.int32), np.array([0, 3], np.uint64), "token ID out of range"),
    ]
    for ids, off, msg in cases:
        with pytest.raises(eg2.ExecutorError, match="KFD: .*" + msg):
            executor.batch(ids, off)
    out = executor.batch(ok_ids, np.array([0, 3], np.uint64))
    assert np.isfinite(out).all()


def test_max_wave_and_single_token(executor, syn):
    ids, off = syn.wave((2046,), seed=51)
    out = executor.batch(ids, off)
    assert np.isfinite(out).all()
    out1 = executor.batch(np.array([7], np.int32), np.array([0, 1], np.uint64))
    assert np.isfinite(out1).all() and abs(np.linalg.norm(out1) - 1) < 1e-5


def test_restatement_live(executor, port, model_baseline, syn):
    """The live restatement (scalar tier) on a fresh mixed wave."""
    import oracle
    ids, off = syn.wave((5, 40, 90), seed=61)
    ref = port.embed(oracle.Gguf(model_baseline), ids, off)
    out = executor.batch(ids, off)
    c = cosine(out, ref)
    print("live restatement cos", c)
    assert c.min() >= 0.997  # measured 0.99764 - 0.0006 (a 5-token sequence: few tokens to average over)


def test_parity_mode_reproduces_restatement(eg2, model_baseline, port, syn):
    """EG2_B200_EXACT (eg2_b200_create): every operation in the reference CPU
    graph's float order -- scalar-tile GEMM rounding, exact-order attention with
    the C library's expf, exact-order PLE projection, and the x86 tiers'
    quantizer and GELU that the fast path also uses.  The embeddings equal the
    restatement run with those choices bit for bit, on config 0 and on a ragged
    wave with a 300-token sequence (sliding window active)."""
    import oracle
    m = eg2.GGUFModel(model_baseline)
    ex = eg2.Gemma2Executor(m, 0, exact=True)
    try:
        g = golden("golden_baseline.npz")
        G = oracle.Gguf(model_baseline)
        for ids, off in ((g["ids"], g["offsets"]), syn.wave((5, 300, 40), seed=90)):
            ref = port.embed(G, ids, off, quant_mode=port.ROUND_X86, gelu_mode=1)
            out = ex.batch(ids, off)
            np.testing.assert_array_equal(out, ref)
        # against the reference's own tiers: inside the north-star tolerance of
        # the scalar tier it shares every float order with except the quantizer
        # rounding and the GELU polynomial
        out = ex.batch(g["ids"], g["offsets"])
        c = cosine(out, g["embed_scalar"])
        print("parity mode vs scalar tier cos", c, "max abs", np.abs(out - g["embed_scalar"]).max())
    finally:
        ex.close()
        m.close()


@pytest.mark.parametrize("norm", ["baseline", "plus1"])
def test_parity_mode_scalar_tier_equals_reference(eg2, syn, norm, port):
    """Parity mode with the scalar tier's quantizer rounding and tanhf GELU
    (EG2_B200_EXACT | EG2_B200_SCALAR_TIER): the embeddings equal, bit for bit,
    the reference's own scalar tier (EI_GEMMA2_CPU_X86=scalar, compiled from its
    sources; golden fixtures) -- on the BASELINE model and on the 1 + N(0, 0.1)
    model whose reference tiers disagree entirely -- and the live restatement
    on a ragged wave."""
    import oracle
    path = syn.model_path(1234, norm)
    m = eg2.GGUFModel(path)
    ex = eg2.Gemma2Executor(m, 0, exact=True, tier="scalar")
    try:
        g = golden(f"golden_{norm}.npz")
        np.testing.assert_array_equal(ex.batch(g["ids"], g["offsets"]), g["embed_scalar"])
        if norm == "baseline":
            ids, off = syn.wave((5, 300, 40), seed=91)
            np.testing.assert_array_equal(ex.batch(ids, off), port.embed(oracle.Gguf(path), ids, off))
    finally:
        ex.close()
        m.close()


@pytest.mark.parametrize("norm", ["baseline", "plus1"])
def test_parity_mode_vnni512_tier_equals_reference_default_tier(eg2, syn, norm):
    """Parity mode at the VNNI-512 tier (EG2_B200_EXACT | EG2_B200_VNNI512_TIER):
    the embeddings equal, bit for bit, the reference CPU graph's DEFAULT tier as
    it runs on an AVX-512 VNNI host (vnni512+gemm512, the tier every golden
    fixture records; compiled from the reference's sources) -- config 0 on both
    weight models, the plus-one model included where the reference's own tiers
    decorrelate; waves of 8, 7 and 3 tokens (its 4-row Q8 tile) and of 9 (its
    512-bit GEMM); the 2 x 128 and 1 x 2048 waves; and the input-rows wave."""
    m = eg2.GGUFModel(syn.model_path(1234, norm))
    ex = eg2.Gemma2Executor(m, 0, exact=True, tier="vnni512")
    try:
        g = golden(f"golden_{norm}.npz")
        assert str(g["best_tier"]) == "vnni512+gemm512"
        np.testing.assert_array_equal(ex.batch(g["ids"], g["offsets"]), g["embed_best"])
        if norm == "baseline":
            s = golden("golden_short_baseline.npz")
            for i in range(4):
                np.testing.assert_array_equal(ex.batch(s[f"ids{i}"], s[f"offsets{i}"]), s[f"embed{i}"])
            lg = golden("golden_long_baseline.npz")
            assert str(lg["tier"]) == "vnni512+gemm512"
            np.testing.assert_array_equal(ex.batch(lg["w2x128_ids"], lg["w2x128_offsets"]), lg["w2x128_embed"])
            np.testing.assert_array_equal(ex.batch(lg["long_ids"], lg["long_offsets"]), lg["long_embed"])
            r = golden("golden_inputs_baseline.npz")
            np.testing.assert_array_equal(ex.batch_rows(r["inputs"], r["offsets"]), r["embed_best"])
    finally:
        ex.close()
        m.close()


def _embedding_rows(model_path, ids):
    """x = (d * q) * sqrt(512) for each id, in float32 exactly as the embed
    kernel and the reference compute it (gemma2_fast.c:942-950)."""
    import oracle
    raw = np.asarray(oracle.Gguf(model_path).raw("token_embd.weight"))
    blk = raw.reshape(262144, 16, 34)[np.asarray(ids)]
    d = np.ascontiguousarray(blk[:, :, :2]).view(np.float16)[..., 0].astype(np.float32)
    q = np.ascontiguousarray(blk[:, :, 2:]).view(np.int8).astype(np.float32)
    return ((d[:, :, None] * q) * np.float32(np.sqrt(np.float32(512)))).astype(np.float32).reshape(len(ids), 512)


def test_input_rows_of_token_embeddings_equal_ids_path(executor, model_baseline, syn):
    """Media soft-token form (512-wide input rows instead of ids,
    gemma2_fast.c:940-941): given exactly the rows the embedding lookup produces,
    the wave is bit-identical to the ids wave, through the monolithic, staged
    and pipelined calls."""
    g = golden("golden_baseline.npz")
    for ids, off in ((g["ids"], g["offsets"]), syn.wave((5, 300, 40, 1), seed=92), syn.wave((600, 700, 1), seed=95)):
        rows = _embedding_rows(model_baseline, ids)
        ref = executor.batch(ids, off)
        np.testing.assert_array_equal(executor.batch_rows(rows, off), ref)
        np.testing.assert_array_equal(executor.collect(executor.submit_rows(rows, off)), ref)
        executor.stage_rows(rows, off)
        executor.launch(3)  # replays start from the uploaded rows every time
        np.testing.assert_array_equal(executor.finish(), ref)


def test_input_rows_match_reference(eg2, executor, model_baseline, port):
    """Random N(0, 1) input rows (golden_inputs_baseline.npz from the reference's
    own CPU graph with ids NULL): within the reference's inter-tier agreement in
    the fast path, and bit-identical to its scalar tier in parity mode with the
    scalar tier's choices."""
    import oracle
    g = golden("golden_inputs_baseline.npz")
    out = executor.batch_rows(g["inputs"], g["offsets"])
    floor = _floor(g)
    c = cosine(out, g["embed_scalar"])
    print("input rows cos vs scalar tier", c, "reference inter-tier", floor)
    assert c.min() >= floor - MARGIN
    m = eg2.GGUFModel(model_baseline)
    px = eg2.Gemma2Executor(m, 0, exact=True, tier="scalar")
    try:
        np.testing.assert_array_equal(px.batch_rows(g["inputs"], g["offsets"]), g["embed_scalar"])
        rng = np.random.default_rng(93)
        off = np.array([0, 70, 71, 333], np.uint64)
        rows = rng.standard_normal((333, 512)).astype(np.float32) * 0.7
        np.testing.assert_array_equal(px.batch_rows(rows, off),
                                      port.embed_inputs(oracle.Gguf(model_baseline), rows, off,
                                                        quant_mode=port.ROUND_SCALAR, gelu_mode=0))
    finally:
        px.close()
        m.close()


def test_input_rows_errors(eg2, executor):
    """Offsets are checked as for ids, with the same messages."""
    rows = np.zeros((4, 512), np.float32)
    with pytest.raises(eg2.ExecutorError, match="invalid KFD sequence offsets"):
        executor.batch_rows(rows, np.array([0, 2, 2, 4], np.uint64))
    with pytest.raises(eg2.ExecutorError, match="1..2048 packed tokens"):
        executor.batch_rows(np.zeros((2049, 512), np.float32), np.array([0, 2049], np.uint64))
    with pytest.raises(eg2.ExecutorError, match="512 wide"):
        executor.batch_rows(np.zeros((4, 100), np.float32), np.array([0, 4], np.uint64))


@pytest.fixture(scope="module")
def wide_executor(eg2, model_baseline):
    m = eg2.GGUFModel(model_baseline)
    ex = eg2.Gemma2Executor(m, 0, max_tokens=8192)
    yield ex
    ex.close()
    m.close()


def test_wide_wave_matches_reference(wide_executor):
    """EG2_B200_WAVE_8192: one 8192-token sequence (the reference CPU graph's
    wave limit, gemma2_fast.c:924) against that graph's own output."""
    g = golden("golden_wide_baseline.npz")
    out = wide_executor.batch(g["ids"], g["offsets"])
    c = float(cosine(out[0], g["embed_best"][0]))
    print("1x8192 cos", c)
    assert c >= 0.9999  # the north star; measured 0.99998


def test_wide_wave_packed_equals_standard_context(wide_executor, executor, syn, model_baseline):
    """A 7600-token wave in an 8192-token context: each sequence's embedding is
    bit-identical to the same sequence alone in a 2048-token context, for ids
    and for input rows."""
    ids, off = syn.wave((2046, 1500, 2046, 2000), seed=94)
    packed = wide_executor.batch(ids, off)
    for s in range(len(off) - 1):
        a, b = int(off[s]), int(off[s + 1])
        solo = executor.batch(ids[a:b], np.array([0, b - a], np.uint64))
        np.testing.assert_array_equal(packed[s], solo[0])
    rows = _embedding_rows(model_baseline, ids)
    np.testing.assert_array_equal(wide_executor.batch_rows(rows, off), packed)


def test_wide_wave_limits(eg2, wide_executor, model_baseline):
    """Past 8192 tokens the CPU graph's own message; parity mode stays at 2048."""
    ids = np.zeros(8193, np.int32)
    with pytest.raises(eg2.ExecutorError, match="accepts 1..8192 input tokens"):
        wide_executor.batch(ids, np.array([0, 8193], np.uint64))
    m = eg2.GGUFModel(model_baseline)
    try:
        with pytest.raises(eg2.ExecutorError, match="up to 2048 tokens"):
            eg2.Gemma2Executor(m, 0, exact=True, max_tokens=8192)
    finally:
        m.close()
