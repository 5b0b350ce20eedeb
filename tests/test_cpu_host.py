"""Host-side logic that needs no GPU: synthetic workloads, the Matryoshka
summation order, the benchmark's accounting, and the N>1 plumbing over gloo."""
import importlib
import json
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT


def test_wave_layout(syn):
    ids, off = syn.wave(syn.CONFIG1_BODIES, seed=100)
    assert ids.dtype == np.int32 and off.dtype == np.uint64
    assert off[0] == 0 and off[-1] == 2048 and len(off) == 17
    for s in range(16):
        seq = ids[off[s]:off[s + 1]]
        assert seq[0] == syn.BOS and seq[-1] == syn.EOS and len(seq) == 128
        assert ((seq[1:-1] >= 3) & (seq[1:-1] < syn.N_VOCAB)).all()
    ids2, off2 = syn.wave(syn.CONFIG1_BODIES, seed=100)
    assert np.array_equal(ids, ids2) and np.array_equal(off, off2)
    empty, eoff = syn.wave((0,))
    assert list(empty) == [syn.BOS, syn.EOS] and list(eoff) == [0, 2]


def test_mixed_load_bounds(syn):
    lens, dims = syn.mixed_load(64, 16)
    assert lens.shape == (64, 16) and (lens + 2 >= 4).all() and (lens + 2 <= 2048).all()
    assert set(np.unique(dims)) <= {128, 256, 512, 768}


def test_sum_squares_order_is_the_servers(eg2):
    """eg2_b200_normalize_prefix (host C) sums squares with two 4-lane
    accumulators over 8-element chunks, then (v0 + v2) + (v1 + v3)
    (kernels.c:35-39,82-93), and scales by 1 / sqrtf(ss); checked against a
    plain float32 restatement at every prefix width."""
    rng = np.random.default_rng(3)
    for _ in range(20):
        emb = (rng.standard_normal(768) * rng.uniform(0.1, 4)).astype(np.float32)
        for n in (128, 256, 512):
            row = emb[:n]
            lanes = [np.float32(0)] * 8
            for c in range(n // 8):
                for i in range(8):
                    lanes[i] = np.float32(lanes[i] + np.float32(row[8 * c + i] * row[8 * c + i]))
            v = [np.float32(lanes[i] + lanes[4 + i]) for i in range(4)]
            ss = np.float32(np.float32(v[0] + v[2]) + np.float32(v[1] + v[3]))
            expect = (row * np.float32(np.float32(1.0) / np.sqrt(ss, dtype=np.float32))).astype(np.float32)
            np.testing.assert_array_equal(eg2.normalize_prefix(emb, n), expect)


def test_normalize_prefix_rejects_other_sizes(eg2):
    with pytest.raises(ValueError):
        eg2.normalize_prefix(np.ones(768, np.float32), 300)


def test_bench_gemm_op_count():
    sys.path.insert(0, ROOT)
    bench = importlib.import_module("bench")
    per_tok = bench.q8_gemm_ops(1) / 2
    local = 512 * (4 * 256 + 1024) + 4 * 256 * 512 + 512 * 4096 + 2048 * 512 + 2 * 512 * 512
    glob = 512 * (4 * 512 + 1024) + 4 * 512 * 512 + 512 * 4096 + 2048 * 512 + 2 * 512 * 512
    assert per_tok == 20 * local + 4 * glob + 512 * 768
    assert bench.whole_job_rate(2048, 4, 10, 100.0) == pytest.approx(2048 * 4 * 10 / 0.1)


def test_bench_attention_pair_count():
    """Algorithmic attention work of bench.py config 5: (query, key) pairs per
    layer, window +-w inside each sequence or (window 0) the whole sequence."""
    sys.path.insert(0, ROOT)
    bench = importlib.import_module("bench")

    def brute(lengths, w):
        return sum(sum(1 for t in range(L) for k in range(L) if not w or abs(t - k) <= w) for L in lengths)

    for lengths, w in (((5,), 1), ((7, 3, 40), 4), ((9, 16), 0), ((128,) * 3, 512)):
        assert bench.attn_pairs(lengths, w) == brute(lengths, w)
    assert bench.attn_pairs((2048,), 0) == 2048 * 2048


def test_bench_reference_arm_contract():
    """`bench.py --impl reference` prints one JSON line with the fields the
    driver reads (config 5: the C restatement of attention_rows, CPU only)."""
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--config", "5"],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "dtype", "config", "impl", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["value"] > 0
    assert {"value", "unit", "cores", "kind", "sample"} <= set(line["cpu_baseline"])
    assert {"value", "unit", "h2d_bytes_per_step", "d2h_bytes_per_step"} <= set(line["e2e"])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    sys.path.insert(0, ROOT)
    bench = importlib.import_module("bench")
    r, w, _ = bench.dist_init("gloo")
    assert (r, w) == (rank, world)
    ids, off = bench.rank_wave(bench.CONFIGS[1][1], r)
    bench.barrier(w)
    fake_ms = 10.0 * (r + 1)  # each rank's device time
    ms_max = bench.reduce_max(fake_ms, w, "cpu")
    rate = bench.whole_job_rate(int(off[-1]), w, 5, ms_max)
    with open(os.path.join(out_dir, f"rank{r}.json"), "w") as f:
        json.dump({"ms_max": ms_max, "rate": rate, "tokens": int(off[-1]), "ids_sum": int(ids.sum())}, f)
    bench.finalize(w)


def test_two_rank_replicas_over_gloo(tmp_path):
    """world_size 2: each rank stages its own full wave, the group only carries
    the barrier and the max-over-ranks time; the whole-job rate counts both ranks'
    tokens over the slowest rank's time."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    res = [json.load(open(tmp_path / f"rank{r}.json")) for r in range(2)]
    assert res[0]["ms_max"] == res[1]["ms_max"] == 20.0
    assert res[0]["tokens"] == res[1]["tokens"] == 2048
    assert res[0]["ids_sum"] != res[1]["ids_sum"]  # distinct waves per rank
    assert res[0]["rate"] == pytest.approx(2 * 2048 * 5 / 0.020)


def test_reference_arm_line(tmp_path):
    """`bench.py --impl reference` prints one JSON line with the contract's keys
    (config 0 keeps it short); it needs the reference build in oracle/_ref."""
    if not os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libeg2ref.so")):
        pytest.skip("oracle/_ref not built")
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--config", "0",
                          "--steps", "1", "--warmup", "0"], capture_output=True, text=True, check=True,
                         timeout=600, cwd=str(tmp_path))
    line = json.loads(out.stdout.strip().splitlines()[-1])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "config",
              "cpu_baseline", "e2e"):
        assert k in line, k
    assert line["impl"] == "reference" and line["value"] > 0 and line["warmup"] >= 3
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "reference"


def test_vnni512_tier_is_a_parity_mode_tier(eg2, model_baseline):
    """tier="vnni512" (EG2_B200_VNNI512_TIER) reproduces a CPU tier's float
    orders and exists only in parity mode; the check precedes any device work."""
    m = eg2.GGUFModel(model_baseline)
    try:
        with pytest.raises(ValueError, match="parity-mode tier"):
            eg2.Gemma2Executor(m, 0, exact=False, tier="vnni512")
        with pytest.raises(ValueError, match="tier must be"):
            eg2.Gemma2Executor(m, 0, exact=True, tier="avx2")
    finally:
        m.close()


def test_http_texts_have_the_packed_lengths(syn):
    """bench.py's HTTP load: with the seeded model's byte-level placeholder
    tokenizer a text of c characters is 4 + c tokens (BOS, the leading U+2581
    as three byte tokens, one token per byte), so each text carries its
    config-3 packed length (body + 2) whenever the body has at least 3 tokens;
    no two texts repeat (the server's response cache is off anyway)."""
    import bench
    lens, _ = syn.mixed_load(256, 16)
    texts = bench.http_texts(lens)
    flat = [t for row in texts for t in row]
    assert len(flat) == 4096 and all(t.isascii() and " " not in t for t in flat)
    for r in range(len(lens)):
        for j, body in enumerate(lens[r]):
            if body >= 3:
                assert 4 + len(texts[r][j]) == int(body) + 2
    long_texts = [t for t in flat if len(t) >= 12]
    assert len(set(long_texts)) == len(long_texts)
