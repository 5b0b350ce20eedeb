"""Embedded tokens/s of the B200 executor on BASELINE's wave configurations.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 1] [--impl b200|reference]

One step = one packed wave through the whole 24-layer graph on each GPU
(config 1: 16 sequences x 128 tokens = 2048 tokens; config 2: 1 x 2048;
config 0: the 4-sequence parity wave).  Config 3 runs the mixed-length request
load (256 requests x 16 texts, packed into waves) through the executor and
reports tokens/s and request latency; config 4 is the Q8_0 GEMM microbench at
the model's shapes.  Every rank holds its own weight
replica and embeds its own wave (weak scaling, no data-path collective); the
process group only provides the barrier and the max-over-ranks time.

value  -- device time of K graph replays with inputs resident in HBM (two
          waves in flight: replays alternate over the context's two lanes),
          CUDA events on the executor's stream around all K; every wave streams
          151 MB of weights and writes 100 MB of PLE rows, more than the 126 MB
          L2; whole-job tokens / max-rank time.  `serial` beside it: one wave
          at a time with an L2 flush (256 MiB write) between steps.
e2e    -- the same waves through ei_gemma2_kfd_batch with host buffers, called
          from two host threads (ids / bounds / positions H2D and the
          embeddings D2H every call), wall time.
--impl reference runs the reference's own CPU graph (oracle/_ref, compiled
from its sources) on the same workload on the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

METRIC = "embedded tokens/s per box (2048-token waves)"
CONFIGS = {0: ("config0: 4 sequences, bodies 8/17/33/64 + BOS/EOS (130 tokens)", (8, 17, 33, 64)),
           1: ("config1: 16 x 128-token sequences = one 2048-token wave", (126,) * 16),
           2: ("config2: 1 x 2048-token sequence", (2046,)),
           3: ("config3: mixed load, 256 requests x 16 texts, lognormal lengths (median 48), packed waves", None),
           4: ("config4: Q8_0 GEMM microbench at the model's shapes, M = 2048 tokens", None),
           5: ("config5: sliding-window attention microbench (d = 256, window 512) at the config 1 and 2 waves", None),
           6: ("config6: config 1's wave (16 x 128 tokens) given as 512-wide input rows, seeded N(0, 1) "
               "(media soft-token form: ids NULL)", (126,) * 16),
           7: ("config7: one 8192-token wave of 4 x 2048-token sequences (the reference CPU graph's wave limit)",
               (2046,) * 4)}
ROWS_CONFIGS = (6,)
WIDE_CONFIGS = (7,)  # run in an 8192-token context (EG2_B200_WAVE_8192)
METRIC_MIXED = "embedded tokens/s per box (mixed-length requests, executor level)"
METRIC_GEMM = "Q8_0 GEMM TOP/s (model shapes, M = 2048)"
METRIC_ATTN = "local-layer attention TFLOP/s (d = 256, window 512; 16x128 and 1x2048 waves)"
# The arithmetic of the fast path, stage by stage.
DTYPE_FAST = ("int8 Q8_0 GEMMs (exact int32 block sums, fp32 scaling), fp16 attention operands with fp32 "
              "scores/softmax/accumulation, bf16 hi+lo PLE projection with fp32 accumulation, fp32 norms")
DTYPE_REFERENCE = "int8 Q8_0 GEMMs (int32 block sums, fp32 scaling), fp32 everything else (reference CPU graph)"
# (name, sequence lengths) of the attention microbench; algorithmic FLOPs are
# 4 heads x 4 d per (query, key) pair the layer visits.
ATTN_SHAPES = (("16x128", (128,) * 16), ("1x2048", (2048,)))


def attn_pairs(lengths, window=512):
    """(query, key) pairs of one layer over packed sequences (window 0: the
    whole sequence, the global layers)."""
    tot = 0
    for L in lengths:
        if not window:
            tot += L * L
            continue
        t = np.arange(L)
        tot += int((np.minimum(L, t + window + 1) - np.maximum(0, t - window)).sum())
    return tot


def attn_bounds(lengths):
    off = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    lo = np.concatenate([[off[i]] * L for i, L in enumerate(lengths)]).astype(np.uint32)
    hi = np.concatenate([[off[i + 1]] * L for i, L in enumerate(lengths)]).astype(np.uint32)
    return lo, hi


def q8_gemm_ops(n_tokens: int) -> float:
    """Algorithmic int8 ops (2*M*N*K) of the Q8_0 GEMMs for one wave."""
    per_tok = 0
    for l in range(24):
        d = 512 if l % 6 == 5 else 256
        per_tok += 512 * (4 * d + 1024)  # q, k, v
        per_tok += 4 * d * 512           # attn_output
        per_tok += 512 * 4096            # ffn up + gate
        per_tok += 2048 * 512            # ffn_down
        per_tok += 2 * 512 * 512         # inp_gate, proj
    per_tok += 512 * 768                 # output
    return 2.0 * per_tok * n_tokens


# DRAM bytes (read + write) per q8gemm launch, averaged over the 145 GEMM
# launches of one config-1 wave in one ncu capture (cold cache); the command
# and the totals are in profiles/q8gemm_wave_dram.md.
GEMM_DRAM_BYTES_PER_LAUNCH = 3.07e6


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """SM clocks and throttle reasons sampled during the timed region: NVML
    read every 5 ms on a thread (read-only queries; nothing is set), or
    nvidia-smi at 200 ms where NVML is unavailable."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, device: int):
        self.device, self.proc, self.thread, self.rows = device, None, None, []

    def _nvml_loop(self, nv, h):
        bits = [nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap]
        while not self.stop:
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.rows.append((float(sm), float(mx), ["Active" if r & b else "Not Active" for b in bits]))
            except Exception:
                pass
            time.sleep(0.005)

    def __enter__(self):
        self.stop = False
        try:
            import threading
            import pynvml as nv
            nv.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            index = int(vis.split(",")[self.device]) if vis and vis.split(",")[0].isdigit() else self.device
            h = nv.nvmlDeviceGetHandleByIndex(index)
            self.thread = threading.Thread(target=self._nvml_loop, args=(nv, h), daemon=True)
            self.thread.start()
            self.source = "nvml 5 ms"
            return self
        except Exception:
            self.thread = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.source = "nvidia-smi 200 ms"
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.thread:
            self.stop = True
            self.thread.join(timeout=5)
        if self.proc:
            time.sleep(0.3)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            for l in out.splitlines():
                f = [x.strip() for x in l.split(",")]
                if len(f) >= 9:
                    try:
                        self.rows.append((float(f[1]), float(f[2]), f[5:9]))
                    except ValueError:
                        pass

    def summary(self):
        rows = self.rows
        if not rows:
            return None
        reasons = sorted({self.NAMES[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows), "source": getattr(self, "source", None)}


def wave_rows(n, seed):
    """Soft-token waves: seeded N(0, 1) input rows [n][512]."""
    return np.random.default_rng(seed).standard_normal((n, 512)).astype(np.float32)


def cpu_baseline_run(model_path, lengths, steps, warmup, seed, rows=False):
    """The reference's own CPU graph (oracle/_ref) on the same waves (with
    rows: the same offsets, the graph started from input rows, ids NULL)."""
    import oracle
    syn = importlib.import_module("embeddinggemma2-amdkfd_b200.synthetic")
    ids, off = syn.wave(lengths, seed=seed)
    ref = oracle.RefGraph(model_path, 0)
    x = wave_rows(int(off[-1]), seed) if rows else None
    run = (lambda: ref.embed_inputs(x, off)) if rows else (lambda: ref.embed(ids, off))
    for _ in range(warmup):
        run()
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    n = int(off[-1])
    med = statistics.median(times)
    res = {"value": n / med, "unit": "tokens/s", "cores": ref.threads, "kind": "reference",
           "tier": ref.tier,
           "sample": f"{len(lengths)} x {n // len(lengths)}-token wave ({n} tokens), median of {steps} after "
                     f"{warmup} warm-up, ei_gemma2_embed_batch_fast_ctx with {ref.threads} threads"}
    ref.close()
    return res


def wave_config(args, desc, n, batch, world):
    """The `config` object of a wave configuration's line, identical in both arms."""
    return {"workload": desc, "model": "EmbeddingGemma 2 text graph, seeded synthetic GGUF (seed 1234, "
            "BASELINE weight distributions)", "tokens_per_wave_per_gpu": n, "sequences_per_wave": batch,
            "parallelism": f"replicas x{world} (whole waves per GPU, no collective)",
            "l2": "inputs larger than L2: each wave streams 151 MB of weights and writes 100 MB of PLE rows "
                  "(L2 126 MB); the serial figure also writes 256 MiB between steps"}


# (name, sequence bodies) of the GPU comparison: the reference CUDA bench's
# headline cases 128x16, 2048x1 and 8192x1 (bench_gemma2_cuda.c:24-25).
GPU_REF_CASES = (("128x16", (126,) * 16), ("2048x1", (2046,)), ("8192x1", (8190,)))


def gpu_baseline_run(eg2, model, model_path, local):
    """The reference's own CUDA executor for this graph (gemma2_cuda.cu +
    cuBLAS, compiled from its sources into oracle/_ref/libeg2cudaref.so) beside
    this executor on the same waves and GGUF, both timed the way the
    reference's bench_gemma2_cuda.c times its own (:69-78): median wall time of
    9 synchronous packed-wave calls (host buffers in and out) after 2 warm-up
    calls.  A reference baseline leg like cpu_baseline: nothing of the
    reference runs inside `value` or `e2e`."""
    import oracle
    syn = eg2.synthetic
    try:
        ref = oracle.CudaRef(model_path, local)
    except (OSError, RuntimeError) as e:
        return {"unavailable": f"reference CUDA executor not loadable: {e}"}

    def median_ms(fn):
        for _ in range(2):
            fn()
        t = []
        for _ in range(9):
            t0 = time.perf_counter()
            fn()
            t.append((time.perf_counter() - t0) * 1000.0)
        return statistics.median(t)

    cases = {}
    try:
        for name, bodies in GPU_REF_CASES:
            ids, off = syn.wave(bodies, seed=300)
            n = int(off[-1])
            ex = eg2.Gemma2Executor(model, local, max_tokens=8192 if n > 2048 else 2048)
            try:
                ours, theirs = ex.batch(ids, off), ref.embed(ids, off)
                ms_b200 = median_ms(lambda: ex.batch(ids, off))
            finally:
                ex.close()
            ms_ref = median_ms(lambda: ref.embed(ids, off))
            a, b = ours.astype(np.float64), theirs.astype(np.float64)
            cos = float(((a * b).sum(1) / np.sqrt((a * a).sum(1) * (b * b).sum(1))).min())
            cases[name] = {"tokens": n, "ref_ms": round(ms_ref, 3), "ref_tokens_s": round(n / ms_ref * 1e3),
                           "b200_ms": round(ms_b200, 3), "b200_tokens_s": round(n / ms_b200 * 1e3),
                           "b200_speedup": round(ms_ref / ms_b200, 3), "min_cosine_b200_vs_ref": round(cos, 6)}
        # Two callers, two waves in flight: the reference executor through its
        # context and one pipeline-slot clone (each its own stream), this one
        # through one context (two lanes); 2 x 40 calls of the 128 x 16 wave.
        ids, off = syn.wave(GPU_REF_CASES[0][1], seed=300)
        n = int(off[-1])
        ref.open_slot()
        ex = eg2.Gemma2Executor(model, local)
        try:
            def two_callers(a, b, calls=40):
                for f in (a, b):
                    f()
                ths = [threading.Thread(target=lambda f=f: [f() for _ in range(calls)]) for f in (a, b)]
                t0 = time.perf_counter()
                for th in ths:
                    th.start()
                for th in ths:
                    th.join()
                return (time.perf_counter() - t0) * 1000.0 / (2 * calls)
            ms_ref2 = two_callers(lambda: ref.embed(ids, off), lambda: ref.embed_slot(ids, off))
            ms_b2 = two_callers(lambda: ex.batch(ids, off), lambda: ex.batch(ids, off))
        finally:
            ex.close()
        cases["128x16_two_callers"] = {"tokens": n, "ref_ms_per_wave": round(ms_ref2, 3),
                                       "ref_tokens_s": round(n / ms_ref2 * 1e3), "b200_ms_per_wave": round(ms_b2, 3),
                                       "b200_tokens_s": round(n / ms_b2 * 1e3),
                                       "b200_speedup": round(ms_ref2 / ms_b2, 3)}
    finally:
        ref.close()
    return {"kind": "reference", "impl": "vendor/embeddinggemma.c/src/gemma2_cuda.cu (cuBLAS GemmEx fp16, mma.sync "
            "flash attention, CUDA graphs), compiled from the reference's sources for sm_100",
            "method": "median wall time of 9 synchronous packed-wave calls after 2 warm-up, host buffers "
                      "(bench_gemma2_cuda.c:69-78); this executor through ei_gemma2_kfd_batch the same way; "
                      "128x16_two_callers: two host threads x 40 calls, the reference through its context and a "
                      "pipeline-slot clone (ei_gemma2_cuda_clone), this executor through one context",
            "cases": cases}


def dist_init(backend="nccl"):
    """One process per GPU (torchrun env); the group carries only the barrier and
    the max-over-ranks time, never embedding data."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        kw = {}
        if backend == "nccl":
            import torch
            kw["device_id"] = torch.device(f"cuda:{local}")
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120), **kw)
    return rank, world, local


def rank_wave(lengths, rank):
    """Each rank embeds its own wave of the same shape (weak scaling): the units
    are whole waves, so ranks share nothing on the data path."""
    syn = importlib.import_module("embeddinggemma2-amdkfd_b200.synthetic")
    return syn.wave(lengths, seed=100 + rank)


def whole_job_rate(tokens_per_rank, world, steps, ms_max):
    """Tokens all ranks embedded / the slowest rank's time."""
    return tokens_per_rank * world * steps / (ms_max * 1e-3)


def reference_arm_mixed(args):
    """Config 3 on the reference's CPU graph: the first `steps` packed waves of
    rank 0's requests (a bounded sample of the load), tokens / wall time."""
    import oracle
    syn = importlib.import_module("embeddinggemma2-amdkfd_b200.synthetic")
    lens, _ = syn.mixed_load(256, 16)
    waves = pack_waves(lens, list(range(len(lens))))[:max(1, args.steps)]
    ref = oracle.RefGraph(syn.model_path(1234, "baseline"), 0)
    inputs = [wave_inputs(w, seed=1000 + i) for i, w in enumerate(waves)]
    ref.embed(*inputs[0])
    t0 = time.perf_counter()
    for ids, off in inputs:
        ref.embed(ids, off)
    sec = time.perf_counter() - t0
    tokens = sum(int(off[-1]) for _, off in inputs)
    cpu = {"value": tokens / sec, "unit": "tokens/s", "cores": ref.threads, "kind": "reference", "tier": ref.tier,
           "sample": f"first {len(waves)} packed waves of the config-3 load ({tokens} tokens), "
                     f"ei_gemma2_embed_batch_fast_ctx with {ref.threads} threads"}
    ref.close()
    line = {"metric": METRIC_MIXED, "value": cpu["value"], "unit": "tokens/s", "n_gpus": args.gpus, "steps": len(waves),
            "warmup": 1, "ms_per_step": sec * 1e3 / len(waves), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": DTYPE_REFERENCE, "data": "synthetic", "config": {"workload": CONFIGS[3][0]},
            "impl": "reference", "cpu_baseline": cpu,
            "e2e": {"value": cpu["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def reference_arm_gemm(args):
    """Config 4 on the CPU: the restatement of the reference's gemm_q8 (scalar
    C, oracle/eg2_oracle.c) per shape on 64 tokens, scaled to TOP/s."""
    import oracle
    oracle.build(ref=False)
    port = oracle.Port()
    rng = np.random.default_rng(4)
    M, tot_ops, tot_s, rows = 64, 0.0, 0.0, []
    for k, n, name in GEMM_SHAPES:
        xq = rng.integers(-127, 128, size=(M, k), dtype=np.int8)
        wq = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
        xd = np.full((M, k // 32), 0x3C00, np.uint16)
        wd = np.full((n, k // 32), 0x3C00, np.uint16)
        port.gemm_q8(wq, wd, xq, xd)
        t0 = time.perf_counter()
        port.gemm_q8(wq, wd, xq, xd)
        sec = time.perf_counter() - t0
        ops_ = 2.0 * M * n * k
        tot_ops, tot_s = tot_ops + ops_, tot_s + sec
        rows.append({"shape": f"{k}->{n}", "use": name, "top_s": ops_ / sec / 1e12})
    v = tot_ops / tot_s / 1e12
    cpu = {"value": v, "unit": "TOP/s", "cores": 1, "kind": "port",
           "sample": "64 tokens per shape through the scalar C restatement of gemm_q8, one thread"}
    line = {"metric": METRIC_GEMM, "value": v, "unit": "TOP/s", "n_gpus": 1, "steps": 1, "warmup": 1,
            "ms_per_step": tot_s * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 (int32 block sums, fp32 scaling)", "data": "synthetic",
            "config": {"workload": CONFIGS[4][0], "M": M}, "impl": "reference", "cpu_baseline": cpu, "shapes": rows,
            "e2e": {"value": v, "unit": "TOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def reference_arm_attention(args):
    """Config 5 on the CPU: the restatement of the reference's attention_rows
    (scalar C, oracle/eg2_oracle.c, fp32) on the 16x128 wave, one thread."""
    import oracle
    oracle.build(ref=False)
    port = oracle.Port()
    rng = np.random.default_rng(5)
    lengths = ATTN_SHAPES[0][1]
    n = sum(lengths)
    q = rng.standard_normal((n, 4, 256)).astype(np.float32)
    k = (rng.standard_normal((n, 2, 256)) * 0.1).astype(np.float32)
    v = rng.standard_normal((n, 2, 256)).astype(np.float32)
    lo, hi = attn_bounds(lengths)
    t0 = time.perf_counter()
    port.attention(q, k, v, lo, hi, 2, 256, 512)
    sec = time.perf_counter() - t0
    val = 16.0 * 256 * attn_pairs(lengths) / sec / 1e12
    cpu = {"value": val, "unit": "TFLOP/s", "cores": 1, "kind": "port",
           "sample": "one 16x128-token local layer through the scalar C restatement of attention_rows"}
    line = {"metric": METRIC_ATTN, "value": val, "unit": "TFLOP/s", "n_gpus": 1, "steps": 1, "warmup": 0,
            "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "config": {"workload": CONFIGS[5][0], "shape": "16x128"},
            "impl": "reference", "cpu_baseline": cpu,
            "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def reference_arm(args, rank, world):
    if rank != 0:
        return
    if args.config == 5:
        return reference_arm_attention(args)
    if args.config == 3:
        return reference_arm_mixed(args)
    if args.config == 4:
        return reference_arm_gemm(args)
    syn = importlib.import_module("embeddinggemma2-amdkfd_b200.synthetic")
    desc, lengths = CONFIGS[args.config]
    model = syn.model_path(1234, "baseline")
    # A bounded sample: a CPU wave of 2048 tokens takes about 0.7 s on 16
    # threads, so at most 10 waves are timed, after 3 warm-up waves.
    steps, warmup = min(args.steps, 10), min(args.warmup, 3)
    cpu = cpu_baseline_run(model, lengths, steps, warmup, seed=100, rows=args.config in ROWS_CONFIGS)
    n = sum(l + 2 for l in lengths)
    line = {"metric": METRIC, "value": cpu["value"], "unit": "tokens/s", "n_gpus": args.gpus, "steps": steps,
            "warmup": warmup, "ms_per_step": 1000.0 * n / cpu["value"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": DTYPE_REFERENCE, "data": "synthetic",
            "config": wave_config(args, desc, n, len(lengths), world),
            "impl": "reference", "cpu_baseline": cpu,
            "e2e": {"value": cpu["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- config 3
def pack_waves(lens, requests, cap=2048):
    """Texts of the given requests, in order, packed greedily into waves of at
    most cap tokens.  Returns [(request, text, packed_length)] per wave."""
    waves, cur, used = [], [], 0
    for r in requests:
        for j, body in enumerate(lens[r]):
            n = int(body) + 2
            if used + n > cap:
                waves.append(cur)
                cur, used = [], 0
            cur.append((r, j, n))
            used += n
    if cur:
        waves.append(cur)
    return waves


def wave_inputs(wave, seed):
    """Token ids and offsets of a packed wave (BOS + random body + EOS per text)."""
    syn = importlib.import_module("embeddinggemma2-amdkfd_b200.synthetic")
    return syn.wave([n - 2 for _, _, n in wave], seed=seed)


def mixed_load_run(args, rank, world, local):
    """Config 3 at the executor: this rank's requests (r % world == rank), all
    queued at t = 0, packed into waves and embedded with host buffers through
    the two-slot pipelined form of ei_gemma2_kfd_batch, each text truncated to
    its request's dimensions and renormalised (Matryoshka).  A request
    completes when its last text does."""
    import torch
    eg2 = importlib.import_module("embeddinggemma2-amdkfd_b200")
    syn = eg2.synthetic
    lens, dims = syn.mixed_load(256, 16)
    mine = [r for r in range(len(lens)) if r % world == rank]
    waves = pack_waves(lens, mine)
    inputs = [wave_inputs(w, seed=1000 + 7919 * rank + i) for i, w in enumerate(waves)]
    torch.cuda.set_device(local)
    model = eg2.GGUFModel(syn.model_path(1234, "baseline"))
    ex = eg2.Gemma2Executor(model, local)

    def run_all():
        """Two waves in flight (eg2_b200_submit / eg2_b200_collect): the host
        truncates one wave's embeddings while the GPU runs the next."""
        remaining = {r: len(lens[r]) for r in mine}
        done_at, t0 = {}, time.perf_counter()

        def complete(slot, w):
            out = ex.collect(slot)
            now = time.perf_counter()
            for i, (r, _, _) in enumerate(w):
                eg2.normalize_prefix(out[i], int(dims[r]))
                remaining[r] -= 1
                if remaining[r] == 0:
                    done_at[r] = (now - t0) * 1000.0

        pending = None
        for w, (ids, off) in zip(waves, inputs):
            slot = ex.submit(ids, off)
            if pending:
                complete(*pending)
            pending = (slot, w)
        if pending:
            complete(*pending)
        return (time.perf_counter() - t0) * 1000.0, done_at

    run_all()  # warm-up: captures the CUDA graph of every bucket the load uses
    barrier(world)
    with ClockSampler(local) as clocks:
        ms, done_at = run_all()
    barrier(world)
    ms_max = reduce_max(ms, world, f"cuda:{local}")
    tokens = sum(n for w in waves for _, _, n in w)
    lat = list(done_at.values())
    if world > 1:
        import torch.distributed as dist
        tot = torch.tensor([float(tokens)], device=f"cuda:{local}")
        dist.all_reduce(tot)
        tokens = int(tot.item())
        gathered = [None] * world
        dist.all_gather_object(gathered, lat)
        lat = [x for g in gathered for x in g]
    line = {"metric": METRIC_MIXED, "value": tokens / (ms_max * 1e-3), "unit": "tokens/s", "n_gpus": world,
            "steps": 1, "warmup": 1, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": DTYPE_FAST, "data": "synthetic",
            "config": {"workload": CONFIGS[3][0], "requests": len(lens), "texts_per_request": len(lens[0]),
                       "tokens": tokens, "waves_per_rank": len(waves),
                       "arrival": "all requests queued at t = 0 (offline load); one executor per GPU",
                       "parallelism": f"replicas x{world}, request r served by rank r % {world}"},
            "latency_ms": {"p50": float(np.percentile(lat, 50)), "p99": float(np.percentile(lat, 99)),
                           "max": float(max(lat))},
            "clocks": clocks.summary()}
    if rank == 0:
        print(json.dumps(line), flush=True)
    del ex
    model.close()


def engine_run(args):
    """Config 3 the way the reference server would run this executor on a box
    of N GPUs once its one-executor limit for this backend is lifted
    (engine.c:1160-1268, slot picking in inference_service.c:171-218): ONE
    process, one ei_gemma2_kfd_create_on context per GPU, one host thread per
    context.  All 256 requests are queued at t = 0 and packed in order into
    waves of at most 2048 tokens; wave i goes to GPU i % N.  Each thread keeps
    two waves in flight (eg2_b200_submit / eg2_b200_collect) and truncates each
    text to its request's dimensions (eg2_b200_normalize_prefix) while the GPU
    runs the next wave.  The ctypes calls release the GIL, so the threads'
    library work runs in parallel; their Python bookkeeping does not.  Per
    thread the wall time splits into submit (validation, staging copy, graph
    launch), collect (waiting for the GPU, result copy) and post (truncation),
    which names the limiter of the 1 -> N curve."""
    import threading
    import torch
    eg2 = importlib.import_module("embeddinggemma2-amdkfd_b200")
    syn = eg2.synthetic
    n_dev = args.gpus
    if torch.cuda.device_count() < n_dev:
        raise SystemExit(f"--engine needs {n_dev} visible GPUs, found {torch.cuda.device_count()}")
    lens, dims = syn.mixed_load(256, 16)
    waves = pack_waves(lens, list(range(len(lens))))
    inputs = [wave_inputs(w, seed=1000 + i) for i, w in enumerate(waves)]
    model = eg2.GGUFModel(syn.model_path(1234, "baseline"))
    exs = [eg2.Gemma2Executor(model, d) for d in range(n_dev)]

    def run_all():
        remaining = {r: len(lens[r]) for r in range(len(lens))}
        done_at, lock = {}, threading.Lock()
        split = [dict(submit=0.0, collect=0.0, post=0.0) for _ in range(n_dev)]
        t0 = time.perf_counter()

        def worker(d):
            ex, acc = exs[d], split[d]
            mine = list(range(d, len(waves), n_dev))

            def complete(slot, w):
                c0 = time.perf_counter()
                out = ex.collect(slot)
                c1 = time.perf_counter()
                finished = []
                for i, (r, _, _) in enumerate(w):
                    eg2.normalize_prefix(out[i], int(dims[r]))
                    finished.append(r)
                c2 = time.perf_counter()
                acc["collect"] += c1 - c0
                acc["post"] += c2 - c1
                with lock:
                    for r in finished:
                        remaining[r] -= 1
                        if remaining[r] == 0:
                            done_at[r] = (c2 - t0) * 1000.0

            pending = None
            for i in mine:
                s0 = time.perf_counter()
                slot = ex.submit(*inputs[i])
                acc["submit"] += time.perf_counter() - s0
                if pending:
                    complete(*pending)
                pending = (slot, waves[i])
            if pending:
                complete(*pending)

        threads = [threading.Thread(target=worker, args=(d,)) for d in range(n_dev)]
        for th in threads:
            th.start()
        for th in threads:
            th.join()
        return (time.perf_counter() - t0) * 1000.0, done_at, split

    run_all()  # warm-up: every context captures the graphs of the buckets the load uses
    with ClockSampler(0) as clocks:
        ms, done_at, split = run_all()
    tokens = sum(n for w in waves for _, _, n in w)
    lat = list(done_at.values())
    line = {"metric": METRIC_MIXED, "value": tokens / (ms * 1e-3), "unit": "tokens/s", "n_gpus": n_dev, "steps": 1,
            "warmup": 1, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": DTYPE_FAST, "data": "synthetic",
            "config": {"workload": CONFIGS[3][0], "requests": len(lens), "texts_per_request": len(lens[0]),
                       "tokens": tokens, "waves": len(waves),
                       "arrival": "all requests queued at t = 0 (offline load)",
                       "parallelism": f"one process, {n_dev} executor contexts, one host thread each, "
                                      f"wave i on GPU i % {n_dev}"},
            "latency_ms": {"p50": float(np.percentile(lat, 50)), "p99": float(np.percentile(lat, 99)),
                           "max": float(max(lat))},
            "thread_split_ms": [{k: round(v * 1000.0, 1) for k, v in sp.items()} for sp in split],
            "clocks_gpu0": clocks.summary()}
    print(json.dumps(line), flush=True)
    for ex in exs:
        ex.close()
    model.close()


# ---------------------------------------------------------------- config 3 over HTTP
SERVER_BIN = os.path.join(ROOT, "oracle", "_ref", "eg2server")
SERVER_CPU_BIN = os.path.join(ROOT, "oracle", "_ref", "eg2server_cpu")
SERVER_CUDA_BIN = os.path.join(ROOT, "oracle", "_ref", "eg2server_cuda")
METRIC_HTTP = "embedded tokens/s per box (mixed-length requests over HTTP)"


def http_texts(lens, salt=""):
    """Texts whose tokenization by the seeded model's placeholder tokenizer has
    each text's packed length (body + 2): it maps every byte of the text, with
    the leading U+2581 (3 bytes), to a byte token after BOS, so a text of c
    characters without spaces is 4 + c tokens.  Each text starts with its own
    (request, text) tag (and salt), so none repeats."""
    texts = []
    for r in range(len(lens)):
        row = []
        for j, body in enumerate(lens[r]):
            c = max(int(body) - 2, 1)
            tag = f"{salt}r{r:x}q{j:x}z"
            row.append((tag + "a" * c)[:c] if c < len(tag) else tag + "a" * (c - len(tag)))
        texts.append(row)
    return texts


def free_port():
    """A TCP port on 127.0.0.1 that nothing listens on right now."""
    import socket
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def start_server(binary, model_path, port, backend, device=None, extra=()):
    env = dict(os.environ)
    if device is not None:
        env["EG2_B200_DEVICE"] = str(device)
    import tempfile
    log_dir = os.environ.get("EG2_B200_SERVER_LOGS") or tempfile.gettempdir()  # where server logs go
    log = open(os.path.join(log_dir, f"server_{backend}_{port}.log"), "w")
    cmd = [binary, "--bind", "127.0.0.1", "--port", str(port), "--backend", backend, "--model", model_path,
           "--text-only", "--response-cache-mb", "0", "--cache-entries", "0", *extra]
    proc = subprocess.Popen(cmd, stdout=log, stderr=subprocess.STDOUT, env=env)
    import http.client
    t0 = time.time()
    while time.time() - t0 < 180:
        if proc.poll() is not None:
            raise RuntimeError(f"server exited with {proc.returncode}: {' '.join(cmd)}")
        try:
            c = http.client.HTTPConnection("127.0.0.1", port, timeout=2)
            c.request("GET", "/healthz")
            if c.getresponse().status == 200:
                c.close()
                return proc
        except OSError:
            time.sleep(0.5)
    proc.kill()
    raise RuntimeError("server did not come up")


def stop_server(proc):
    proc.terminate()
    try:
        proc.wait(timeout=30)
    except subprocess.TimeoutExpired:
        proc.kill()
        proc.wait()


def http_embed(conn, texts, dims):
    """One /api/embed request (base64 float32 rows); returns the embeddings."""
    import base64
    body = json.dumps({"input": texts, "dimensions": int(dims), "encoding_format": "base64"}).encode()
    conn.request("POST", "/api/embed", body=body, headers={"Content-Type": "application/json"})
    resp = conn.getresponse()
    payload = resp.read()
    if resp.status != 200:
        raise RuntimeError(f"HTTP {resp.status}: {payload[:200]!r}")
    rows = json.loads(payload)["embeddings"]
    return np.stack([np.frombuffer(base64.b64decode(r), np.float32) for r in rows])


def _http_client(job):
    """Client process of http_run: `threads` keep-alive connections to the
    server on `port` take its requests in order; returns {request: ms from the
    common start}."""
    import http.client
    import queue
    import threading
    port, requests, threads, start, salt = job
    syn = importlib.import_module("embeddinggemma2-amdkfd_b200.synthetic")
    lens, dims = syn.mixed_load(256, 16)
    texts = http_texts(lens, salt)
    jobs = queue.Queue()
    for r in requests:
        jobs.put(r)
    done_at, lock = {}, threading.Lock()
    conns = [http.client.HTTPConnection("127.0.0.1", port, timeout=600) for _ in range(threads)]
    time.sleep(max(0.0, start - time.time()))

    def client(conn):
        while True:
            try:
                r = jobs.get_nowait()
            except queue.Empty:
                break
            out = http_embed(conn, texts[r], dims[r])
            assert out.shape == (16, int(dims[r])) and np.isfinite(out).all()
            with lock:
                done_at[r] = (time.time() - start) * 1000.0
        conn.close()
    ths = [threading.Thread(target=client, args=(c,)) for c in conns]
    for th in ths:
        th.start()
    for th in ths:
        th.join()
    return done_at


def http_run(args, reference=False):
    """Config 3 over HTTP through the reference's own server
    (vendor/embeddinggemma.c/src/server.c + inference_service.c + engine.c,
    built unchanged by oracle/Makefile `server`): its tokenizer, batcher and
    JSON layer in front of this executor (`--backend kfd`), one server process
    per GPU (the engine allows one KFD executor per process,
    engine.c:1163-1169).  All 256 requests (16 texts each, dims per request)
    are queued at t = 0; one client process per server (32 keep-alive
    connections each) takes them in order, request r on server r % N,
    responses as base64 float32.  tokens/s = the
    requests' packed tokens / wall time; latency from t = 0 to the response.
    --impl reference runs the same server on its own CPU backend (16 threads)
    over the first 16 requests (a bounded sample)."""
    import http.client
    import queue
    import threading
    syn = importlib.import_module("embeddinggemma2-amdkfd_b200.synthetic")
    lens, dims = syn.mixed_load(256, 16)
    texts = http_texts(lens)
    n_req = 16 if reference else len(lens)
    cuda = not reference and args.http_backend == "cuda"
    n_srv = 1 if reference or cuda else args.gpus
    model_path = syn.model_path(1234, "baseline", tokenizer=True)
    binary = SERVER_CPU_BIN if reference else SERVER_CUDA_BIN if cuda else SERVER_BIN
    if not os.path.exists(binary):
        raise SystemExit(f"{binary} missing: make -C oracle server")
    backend = "cpu" if reference else "cuda" if cuda else "kfd"
    # The GPU servers' CPU pool (used only by media towers) is kept small so
    # that N server processes do not crowd the host.
    extra = ("--threads", str(os.cpu_count() or 8)) if reference else ("--threads", "2")
    # One client process per GPU (a single Python client caps out near 2.3M
    # tokens/s), each with 32 keep-alive connections (the CPU arm: 8).
    n_cli = 1 if reference else args.gpus
    conns_per_cli = 8 if reference else 32
    conns_per_srv = conns_per_cli * n_cli // n_srv
    if cuda:  # one process on every GPU, two pipeline slots (waves in flight) per GPU; the server
        # keeps at most 255 keep-alive connections, fewer than its HTTP workers
        extra += ("--cuda-devices", ",".join(str(d) for d in range(args.gpus)), "--pipeline-slots", "2",
                  "--keepalive-connections", str(min(conns_per_srv, 255)),
                  "--workers", str(min(conns_per_srv, 255) + 64))
    ports = [free_port() for _ in range(n_srv)]
    procs = [start_server(binary, model_path, ports[d], backend, None if reference or cuda else d, extra)
             for d in range(n_srv)]
    # The client processes are spawned (no CUDA state, each its own GIL) and
    # start at the same wall-clock instant, so request latency is measured
    # from the common t = 0; client c sends requests r % n_cli == c to server
    # c % n_srv.
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    try:
        def run_all(requests, salt=""):
            start = time.time() + 2.0
            work = [(ports[c % n_srv], [r for r in requests if r % n_cli == c], conns_per_cli, start, salt)
                    for c in range(n_cli)]
            with ctx.Pool(n_cli) as pool:
                parts = pool.map(_http_client, work)
            done_at = {r: t for part in parts for r, t in part.items()}
            return max(done_at.values()), done_at

        # Warm-up: the same load with other texts of the same lengths, untimed,
        # so that every wave shape it packs has its CUDA graph (one per
        # 64-token bucket and lane) and no text of the timed run was seen.
        run_all(range(n_req) if not reference else range(2), salt="w")
        ms, done_at = run_all(range(n_req))
    finally:
        for p in procs:
            stop_server(p)
    tokens = int(sum(4 + len(t) for r in range(n_req) for t in texts[r]))  # BOS + U+2581 (3 bytes) + bytes
    lat = list(done_at.values())
    line = {"metric": METRIC_HTTP, "value": tokens / (ms * 1e-3), "unit": "tokens/s", "n_gpus": 0 if reference
            else args.gpus, "steps": 1, "warmup": 1, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": DTYPE_REFERENCE if reference else DTYPE_FAST, "data": "synthetic",
            "config": {"workload": CONFIGS[3][0] + ", over HTTP (/api/embed, base64)", "requests": n_req,
                       "texts_per_request": 16, "tokens": tokens,
                       "server": "reference server.c, " + ("cpu backend" if reference else
                                                           f"cuda backend = this executor through the reference's "
                                                           f"CUDA executor ABI, one process on {args.gpus} GPU(s), "
                                                           "2 pipeline slots per GPU" if cuda else
                                                           f"kfd backend = this executor, {n_srv} process(es), "
                                                           "one per GPU"),
                       "arrival": "all requests queued at t = 0 (offline load)",
                       "client": f"{n_cli} client process(es), {conns_per_cli} keep-alive connections each"},
            "latency_ms": {"p50": float(np.percentile(lat, 50)), "p99": float(np.percentile(lat, 99)),
                           "max": float(max(lat))},
            "e2e": {"value": tokens / (ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0, "api": "HTTP /api/embed"}}
    if reference:
        line["impl"] = "reference"
    else:
        line["tokenizer"] = tokenizer_rate(model_path, [t for row in texts for t in row])
    print(json.dumps(line), flush=True)


def tokenizer_rate(model_path, texts):
    """The reference engine's own tokenizer (tokenizer.c, ei_tokenize_spm as
    engine.c:1143 calls it) over the load's texts on one host thread: the
    per-thread rate that the server's tokenizer workers
    (--tokenizer-workers, inference_service.h:21) multiply."""
    import ctypes as C
    import oracle
    lib = C.CDLL(oracle.ENGINE_LINK_SO)
    lib.eg2link_open_cpu.restype = C.c_void_p
    lib.eg2link_open_cpu.argtypes = [C.c_char_p]
    lib.eg2link_tokenize.restype = C.c_size_t
    lib.eg2link_tokenize.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t, C.c_void_p, C.c_size_t]
    lib.eg2link_close.argtypes = [C.c_void_p]
    h = lib.eg2link_open_cpu(model_path.encode())
    enc = [t.encode() for t in texts]
    tokens = 0
    t0 = time.perf_counter()
    for b in enc:
        tokens += lib.eg2link_tokenize(h, b, len(b), None, 0)
    dt = time.perf_counter() - t0
    lib.eg2link_close(h)
    return {"tokens_per_s_one_thread": tokens / dt, "tokens": tokens, "texts": len(enc),
            "note": "seeded model's placeholder byte-level vocabulary (the real 262k-piece model is not available)"}


# ---------------------------------------------------------------- config 4
GEMM_SHAPES = [(512, 2048, "q|k|v local"), (512, 3072, "q|k|v global"), (1024, 512, "attn_output local"),
               (2048, 512, "attn_output global, ffn_down"), (512, 4096, "ffn gate|up (GeGLU epilogue)"),
               (512, 512, "inp_gate, proj"), (512, 768, "output")]


def gemm_microbench(args, local):
    """Config 4: each Q8_0 GEMM shape of the model at M = 2048 tokens, timed as a
    CUDA graph of `steps` launches (inputs resident, each launch re-reads its
    operands), plus an exactness check of the int32 block sums (unit scales:
    every output is an exact integer sum) against numpy on 64 tokens."""
    import torch
    ops = importlib.import_module("embeddinggemma2-amdkfd_b200.ops")
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    M = 2048
    rng = np.random.default_rng(4)
    pk, src = peaks()
    peak = 2.0 * pk["bf16_tflops"]
    rows, tot_ops, tot_s, exact_all = [], 0.0, 0.0, True
    for k, n, name in GEMM_SHAPES:
        geglu = "GeGLU" in name
        xq = rng.integers(-127, 128, size=(M, k), dtype=np.int8)
        wq = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
        xs1 = torch.ones(k // 32 * M, device=dev)
        ws1 = torch.ones(k // 32 * n, device=dev)
        xt, wt = torch.from_numpy(xq).to(dev), torch.from_numpy(wq).to(dev)
        if geglu:
            q = torch.zeros(M * n // 2, dtype=torch.int8, device=dev)
            sc = torch.zeros(n // 64 * M, device=dev)
            launch = lambda: ops.q8_geglu(q, sc, M, xt, xs1, M, wt, ws1, M, k, n // 2)
        else:
            out = torch.zeros(M * n, device=dev)
            launch = lambda: ops.q8_mm(out, xt, xs1, M, wt, ws1, M, k, n)
            launch()
            torch.cuda.synchronize()
            got = out.view(M, n)[:64].cpu().numpy().astype(np.int64)
            ref = xq[:64].astype(np.int64) @ wq.astype(np.int64).T
            exact = bool(np.array_equal(got, ref))
            exact_all &= exact
        for _ in range(args.warmup):
            launch()
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for _ in range(args.steps):
                    launch()
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1000.0 / args.steps
        ops_ = 2.0 * M * n * k
        tot_ops, tot_s = tot_ops + ops_, tot_s + us * 1e-6
        rows.append({"shape": f"{k}->{n}", "use": name, "us": round(us, 2), "top_s": round(ops_ / us / 1e6, 1),
                     "frac_of_peak": round(ops_ / us / 1e6 / peak, 4),
                     "int32_block_sums_exact": None if geglu else exact})
        del g
    # BF16 PLE projection 512 -> 12288 (fp32 activations split hi + lo).
    x = torch.randn(M, 512, device=dev)
    hi = x.to(torch.bfloat16)
    lo = (x - hi.float()).to(torch.bfloat16)
    w = (torch.randn(12288, 512, device=dev) / 22.6).to(torch.bfloat16)
    nw = torch.ones(512, device=dev)
    ple = torch.zeros(M * 12288, device=dev)
    pl = lambda: ops.ple_proj(ple, hi.view(torch.uint16), lo.view(torch.uint16), w.view(torch.uint16), nw, M)
    for _ in range(args.warmup):
        pl()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        pl()
    e1.record()
    torch.cuda.synchronize()
    ple_us = e0.elapsed_time(e1) * 1000.0 / args.steps
    line = {"metric": METRIC_GEMM, "value": tot_ops / tot_s / 1e12, "unit": "TOP/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": tot_s * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8 (int32 block sums, fp32 scaling)",
            "data": "synthetic", "config": {"workload": CONFIGS[4][0], "M": M},
            "peak": {"value": peak, "unit": "TOP/s", "source": f"2 x bf16_tflops of {src} MEASURED_PEAKS"},
            "int32_block_sums_exact": exact_all, "shapes": rows,
            "ple_bf16": {"shape": "512->12288", "us": round(ple_us, 2),
                         "tflop_s_executed": round(2.0 * 2 * M * 12288 * 512 / ple_us / 1e6, 1),
                         "note": "eager launches; hi + lo halves, so 2x the algorithmic 25.8 GFLOP"}}
    print(json.dumps(line), flush=True)


def attention_microbench(args, local):
    """Config 5: one sliding-window layer's attention (q/k/v fp16, d = 256,
    window 512) on the config 1 and config 2 waves through the tcgen05 kernel
    (eg2_launch_attention_tc) and, for comparison, the mma.sync kernel
    (eg2_launch_attention_f16); each timed as a CUDA graph of `steps` launches
    with inputs resident.  Per shape: one parity launch first (tcgen05 against
    mma.sync, max |difference|), then `warmup` launches, then the graph.  Order
    of fp32-output tcgen05 launches: shape 1 parity, warm-ups, 2 x steps graph
    nodes, then shape 2 likewise (the Q8-output timing of each shape follows
    its mma.sync timing).  The same two waves then run through the global
    layers' form (d = 512, one KV head, no window), reported beside the
    value."""
    import torch
    ops = importlib.import_module("embeddinggemma2-amdkfd_b200.ops")
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    pk, src = peaks()
    peak = pk["bf16_tflops"]
    rng = np.random.default_rng(5)

    def timed(launch):
        for _ in range(args.warmup):
            launch()
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for _ in range(args.steps):
                    launch()
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        del g
        return e0.elapsed_time(e1) * 1000.0 / args.steps

    def measure(name, lengths, d, window):
        n, kv = sum(lengths), 512 // d
        q = torch.from_numpy(rng.standard_normal((n, 4, d)).astype(np.float16)).to(dev)
        k = torch.from_numpy((rng.standard_normal((n, kv, d)) * 0.1 * (256 / d) ** 0.5).astype(np.float16)).to(dev)
        v = torch.from_numpy(rng.standard_normal((n, kv, d)).astype(np.float16)).to(dev)
        lo, hi = attn_bounds(lengths)
        b = torch.from_numpy(np.stack([lo, hi], 1).ravel().copy()).to(dev)
        o_tc, o_mma = torch.zeros(n * 4 * d, device=dev), torch.zeros(n * 4 * d, device=dev)
        q8 = torch.zeros(n * 4 * d, dtype=torch.int8, device=dev)
        q8s = torch.zeros(4 * d // 32 * n, device=dev)
        tc = lambda: ops.attention_tc(o_tc, q, k, v, b, n, window, d)
        tc_q8 = lambda: ops.attention_tc_q8(q8, q8s, n, q, k, v, b, n, window, d=d)
        mma = lambda: ops.attention_f16(o_mma, q, k, v, b, n, d, window)
        tc(), mma()
        torch.cuda.synchronize()
        diff = float((o_tc - o_mma).abs().max())
        us_tc, us_mma = timed(tc), timed(mma)
        us_q8 = timed(tc_q8)
        fl = 16.0 * d * attn_pairs(lengths, window)
        return fl, us_tc, {"shape": name, "d": d, "window": window, "gflop": round(fl / 1e9, 3),
                           "us_tcgen05": round(us_tc, 2), "tflop_s": round(fl / us_tc / 1e6, 1),
                           "frac_of_peak": round(fl / us_tc / 1e6 / peak, 4), "us_mma_sync": round(us_mma, 2),
                           "max_abs_diff_vs_mma_sync": diff, "us_tcgen05_q8_out": round(us_q8, 2)}

    rows, tot_fl, tot_s = [], 0.0, 0.0
    for name, lengths in ATTN_SHAPES:
        fl, us, row = measure(name, lengths, 256, 512)
        tot_fl, tot_s = tot_fl + fl, tot_s + us * 1e-6
        rows.append(row)
    # The global layers (d = 512, one KV head, no window) at the same waves.
    global_rows = [measure(name, lengths, 512, 0)[2] for name, lengths in ATTN_SHAPES]
    line = {"metric": METRIC_ATTN, "value": tot_fl / tot_s / 1e12, "unit": "TFLOP/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": tot_s * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16 (fp32 accumulate and softmax)",
            "data": "synthetic", "config": {"workload": CONFIGS[5][0]},
            "peak": {"value": peak, "unit": "TFLOP/s", "source": f"bf16_tflops of {src} MEASURED_PEAKS"},
            "shapes": rows, "global_layer_shapes": global_rows, "gpu_launches": 2 * len(ATTN_SHAPES) * args.steps,
            "note": "value and tflop_s: fp32 output; us_tcgen05_q8_out: the executor's form, Q8_0 output of the O projection"}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=1, choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity-mode", action="store_true", help="skip the parity-mode measurement")
    ap.add_argument("--engine", action="store_true",
                    help="config 3 in one process: one executor context and host thread per GPU (--gpus of them)")
    ap.add_argument("--no-gpu-baseline", action="store_true",
                    help="skip timing the reference's own CUDA executor beside this one")
    ap.add_argument("--http", action="store_true",
                    help="config 3 over HTTP: the reference's own server (oracle/_ref/eg2server, --backend kfd "
                         "through this executor), one server process per GPU (--gpus of them)")
    ap.add_argument("--http-backend", default="kfd", choices=["kfd", "cuda"],
                    help="with --http: kfd = one server process per GPU through the KFD executor ABI; cuda = ONE "
                         "server process on all --gpus through the reference's CUDA executor ABI "
                         "(--cuda-devices, two pipeline slots per GPU)")
    ap.add_argument("--profile-gpu-reference", action="store_true",
                    help="like --profile-wave, for the reference's own CUDA executor (gemma2_cuda.cu) on the same "
                         "wave: one packed-wave call inside cudaProfilerStart/Stop")
    ap.add_argument("--profile-wave", action="store_true",
                    help="for ncu --profile-from-start off: one wave of --config after warm-up, then plain "
                         "elementwise copies of the row kernels' byte counts, inside cudaProfilerStart/Stop")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank, world, local = dist_init()
    if args.impl == "reference" and not (args.config == 3 and args.http):
        reference_arm(args, rank, world)
        return finalize(world)
    if args.profile_wave or args.profile_gpu_reference:
        if rank == 0:
            (profile_gpu_reference if args.profile_gpu_reference else profile_wave)(args, local)
        return finalize(world)
    if args.config == 3 and args.http:
        if rank == 0:
            http_run(args, reference=args.impl == "reference")
        return finalize(world)
    if args.config == 3 and args.engine:
        if rank == 0:
            engine_run(args)
        return finalize(world)
    if args.config == 3:
        mixed_load_run(args, rank, world, local)
        return finalize(world)
    if args.config == 4:
        if rank == 0:
            gemm_microbench(args, local)
        return finalize(world)
    if args.config == 5:
        if rank == 0:
            attention_microbench(args, local)
        return finalize(world)

    import torch
    eg2 = importlib.import_module("embeddinggemma2-amdkfd_b200")
    syn = eg2.synthetic
    desc, lengths = CONFIGS[args.config]
    model_path = syn.model_path(1234, "baseline")
    torch.cuda.set_device(local)
    model = eg2.GGUFModel(model_path)
    ex = eg2.Gemma2Executor(model, local, max_tokens=8192 if args.config in WIDE_CONFIGS else 2048)
    ids, off = rank_wave(lengths, rank)
    n, batch = int(off[-1]), len(off) - 1
    rows = wave_rows(n, 100 + rank) if args.config in ROWS_CONFIGS else None
    stage = (lambda: ex.stage_rows(rows, off)) if rows is not None else (lambda: ex.stage(ids, off))
    run_batch = (lambda: ex.batch_rows(rows, off)) if rows is not None else (lambda: ex.batch(ids, off))
    cap = 8192 if args.config in WIDE_CONFIGS else 2048
    h2d_bytes = (5 * cap + 2) * 4 + (-(-n // 64) * 64 * 512 * 4 if rows is not None else 0)
    stream = torch.cuda.ExternalStream(ex.stream, device=local)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=local)

    # ---- value: device-resident waves, two in flight (the lanes alternate)
    stage()
    ex.launch(max(args.warmup, 2))
    ex.finish()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            e0.record(stream)
            ex.launch(args.steps)
            e1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    out_dev = ex.finish()
    dev_ms = e0.elapsed_time(e1)
    dev_ms_max = reduce_max(dev_ms, world, f"cuda:{local}")

    # ---- serial: one wave at a time on one lane, L2 flushed between steps
    serial_steps = min(args.steps, 100)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(serial_steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(serial_steps)]
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for i in range(serial_steps):
            flush.zero_()  # L2 flush, outside the timed events
            starts[i].record(stream)
            ex.launch(1)
            ends[i].record(stream)
    torch.cuda.synchronize()
    serial_ms = sum(a.elapsed_time(b) for a, b in zip(starts, ends)) / serial_steps

    # ---- e2e: the public C ABI with host buffers every call, from two host
    # threads (the context runs two calls' waves at once); wall time
    for _ in range(args.warmup):
        run_batch()
    outs = [None, None]
    busy_ms = [[], []]

    def caller(k, count):
        for _ in range(count):
            c0 = time.perf_counter()
            outs[k] = run_batch()
            busy_ms[k].append((time.perf_counter() - c0) * 1000.0)
    barrier(world)
    torch.cuda.synchronize()
    threads = [threading.Thread(target=caller, args=(k, args.steps // 2 + (k < args.steps % 2)))
               for k in range(2)]
    t0 = time.perf_counter()
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    e2e_ms = (time.perf_counter() - t0) * 1000.0
    barrier(world)
    e2e_ms_max = reduce_max(e2e_ms, world, f"cuda:{local}")
    for out in outs:
        assert np.isfinite(out).all() and np.allclose(out, out_dev, atol=1e-6)
    # latency of one call alone (no other call in flight)
    call_ms = []
    for _ in range(min(args.steps, 100)):
        c0 = time.perf_counter()
        run_batch()
        call_ms.append((time.perf_counter() - c0) * 1000.0)
    loaded_ms = busy_ms[0] + busy_ms[1]

    # ---- dominant kernel: per-group event timing of one eager wave
    stage()
    prof = ex.profile()
    gemm_ms = sum(v for k, v in prof.items() if k.startswith("gemm_"))
    pk, src = peaks()
    int8_peak = 2.0 * pk["bf16_tflops_sustained"]
    achieved = q8_gemm_ops(n) / (gemm_ms * 1e-3) / 1e12
    line = {
        "metric": METRIC,
        "value": whole_job_rate(n, world, args.steps, dev_ms_max),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dev_ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": DTYPE_FAST, "data": "synthetic",
        "config": wave_config(args, desc, n, batch, world),
        "e2e": {"value": whole_job_rate(n, world, args.steps, e2e_ms_max), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d_bytes,
                "d2h_bytes_per_step": batch * 768 * 4,
                "api": "ei_gemma2_kfd_batch from two host threads (two calls' waves in flight)"},
        "serial": {"ms_per_step": serial_ms, "value": whole_job_rate(n, 1, 1, serial_ms), "steps": serial_steps,
                   "what": "one wave at a time on one lane, 256 MiB L2 flush between steps, rank 0"},
        "latency_ms": {"p50": float(np.percentile(call_ms, 50)), "p99": float(np.percentile(call_ms, 99)),
                       "loaded_p50": float(np.percentile(loaded_ms, 50)),
                       "loaded_p99": float(np.percentile(loaded_ms, 99)),
                       "what": f"one ei_gemma2_kfd_batch call of the wave ({batch} texts), host buffers, rank {rank}: "
                               "alone (p50/p99) and during the two-thread e2e run (loaded_*)"},
        "gpu_launches": ex.kernels_per_wave * args.steps,
        "roofline": {"kernel": "q8gemm_kernel (all Q8_0 GEMM launches of a wave)", "bound": "tensor",
                     "achieved": achieved, "peak": int8_peak, "unit": "TOP/s", "frac": achieved / int8_peak,
                     "peak_source": f"2 x bf16_tflops_sustained of {src} MEASURED_PEAKS (dense int8 = 2x bf16)",
                     "traffic": GEMM_DRAM_BYTES_PER_LAUNCH,
                     "traffic_note": "dram read+write bytes per launch, ncu capture averaged over one wave's GEMMs"},
        "profile_ms": {k: round(v, 4) for k, v in prof.items()},
    }
    c = clocks.summary()
    line["clocks"] = c
    if rank == 0 and world == 1 and args.config in (0, 1, 2) and not args.no_parity_mode:
        line["parity_mode"] = parity_mode_run(eg2, model, ids, off, args)
    del ex
    if rank == 0 and world == 1 and args.config == 1 and not args.no_gpu_baseline:
        line["gpu_baseline"] = gpu_baseline_run(eg2, model, model_path, local)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_run(model_path, lengths, 3, 1, seed=100,
                                                rows=args.config in ROWS_CONFIGS)
    if rank == 0:
        print(json.dumps(line), flush=True)
    finalize(world)


# Same-size plain copies for the launch list: read + write bytes of post_add
# (13.4 MB), gate_quant (9.4 MB) and qkv_post<256> (25.2 MB) at 2048 tokens.
COPY_FLOOR_MB = (6.7, 4.7, 12.6)


def profile_wave(args, local):
    """One wave of the configuration, after warm-up, between
    cudaProfilerStart and cudaProfilerStop (so that `ncu --profile-from-start
    off` captures exactly its kernels), followed by elementwise copies
    (torch.mul by 1) whose read + write bytes equal those of the row kernels:
    the launch-latency and bandwidth floor of a plain kernel of the same size
    under the same capture."""
    import torch
    eg2 = importlib.import_module("embeddinggemma2-amdkfd_b200")
    desc, lengths = CONFIGS[args.config]
    if lengths is None or args.config in ROWS_CONFIGS or args.config in WIDE_CONFIGS:
        raise SystemExit("--profile-wave takes a token-id wave configuration (0, 1 or 2)")
    torch.cuda.set_device(local)
    model = eg2.GGUFModel(eg2.synthetic.model_path(1234, "baseline"))
    ex = eg2.Gemma2Executor(model, local)
    ids, off = eg2.synthetic.wave(lengths, seed=100)
    ex.stage(ids, off)
    ex.launch(args.warmup)
    ex.finish()
    bufs = []
    for mb in COPY_FLOOR_MB:
        a = torch.randn(int(mb * 1e6) // 4, device=f"cuda:{local}")
        b = torch.empty_like(a)
        torch.mul(a, 1.0, out=b)
        bufs.append((a, b))
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    ex.launch(1)
    ex.finish()
    for a, b in bufs:
        torch.mul(a, 1.0, out=b)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print(json.dumps({"profiled": desc, "kernels_per_wave": ex.kernels_per_wave,
                      "copies_mb_read_plus_write": [2 * mb for mb in COPY_FLOOR_MB]}))
    ex.close()
    model.close()


def profile_gpu_reference(args, local):
    """One packed-wave call of the reference's own CUDA executor
    (oracle/_ref/libeg2cudaref.so) on the configuration's wave, after warm-up,
    between cudaProfilerStart and cudaProfilerStop: its launch list beside this
    executor's (--profile-wave), kernel by kernel."""
    import torch
    import oracle
    syn = importlib.import_module("embeddinggemma2-amdkfd_b200.synthetic")
    desc, lengths = CONFIGS[args.config]
    if lengths is None:
        raise SystemExit("--profile-gpu-reference takes a token-id wave configuration")
    torch.cuda.set_device(local)
    ref = oracle.CudaRef(syn.model_path(1234, "baseline"), local)
    ids, off = syn.wave(lengths, seed=100)
    for _ in range(max(args.warmup, 3)):
        ref.embed(ids, off)
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    ref.embed(ids, off)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    ref.close()
    print(json.dumps({"profiled": desc, "executor": "reference gemma2_cuda.cu"}))


def parity_mode_run(eg2, model, ids, off, args):
    """The same wave in parity mode, whose embeddings are bit-identical to a
    tier of the reference CPU graph: with the scalar tier's choices
    (EG2_B200_EXACT | EG2_B200_SCALAR_TIER), and, under `vnni512_tier`, in the
    float orders of its default tier on an AVX-512 VNNI host (EG2_B200_EXACT |
    EG2_B200_VNNI512_TIER).  Device-resident waves timed with CUDA events like
    `value` (a few steps; a wave takes tens of ms)."""
    import torch
    n = int(off[-1])

    def timed(tier):
        px = eg2.Gemma2Executor(model, 0, exact=True, tier=tier)
        stream = torch.cuda.ExternalStream(px.stream, device=0)
        px.stage(ids, off)
        px.launch(2)
        px.finish()
        steps = max(4, min(args.steps, 10))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            e0.record(stream)
            px.launch(steps)
            e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        px.finish()
        k = px.kernels_per_wave
        px.close()
        return {"value": n / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms, "steps": steps,
                "kernels_per_wave": k}

    res = timed("scalar")
    res.update(dtype="reference scalar tier's float order: int8 Q8_0 GEMMs with the scalar tile's roundings, "
                     "fp32 CUDA-core attention and PLE in the CPU loop order",
               parity="bit-identical to the reference CPU graph's scalar tier (tests/test_gpu_executor.py)")
    v = timed("vnni512")
    v.update(dtype="reference default tier's float order on an AVX-512 VNNI host: Q8_0 GEMMs as its 16-lane "
                   "int32 lane sums with fused multiply-adds (dp4a on CUDA cores), fp32 attention and PLE in its "
                   "8-lane orders",
             parity="bit-identical to the reference CPU graph's default tier, vnni512+gemm512 "
                    "(tests/test_gpu_executor.py, tests/test_gpu_layers.py)")
    res["vnni512_tier"] = v
    return res


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def reduce_max(v, world, device):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def finalize(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
